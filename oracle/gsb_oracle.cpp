// gsb_oracle.cpp -- CPU parity oracle for the gswarp_b200 3DGS hot path.
//
// TEST INFRASTRUCTURE ONLY.  This file is a plain C++ restatement of the
// arithmetic of gswarp v1.1.0 (fancifulland2718/gswarp, Warp kernels) for the
// 3DGS training path.  It exists so that the CUDA kernels of gswarp_b200 can be
// checked against the reference algorithm on identical inputs.  Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg load it; the product
// path never links, loads or calls it.
//
// Build: see oracle/Makefile.  Compiled with -O2 -ffp-contract=off and no fast
// math, so every float expression below is evaluated in IEEE binary32 exactly
// in the order written (the reference's Python/Warp expression order,
// left-to-right).  The CUDA translation units that must agree bit-for-bit
// (preprocess, binning, preprocess backward, KNN) are compiled with
// -fmad=false for the same reason.
//
// Conventions shared with the reference:
//   * view/proj matrices are read as flat 16-float arrays, index [c*4+r]
//     (gswarp/_internal/backends/warp/preprocess_kernels.py:134).
//   * BLOCK_X = BLOCK_Y = 16 (constants.py:6-7).
//   * float->int conversions saturate and map NaN to 0, which is what the
//     CUDA cvt.rzi.s32.f32 instruction (used by Warp's wp.int32()) does.
//   * The only transcendental on an integer-determining path is the AccuTile
//     opacity threshold 2*log(max(255*op,1)).  Both this oracle and the CUDA
//     kernels evaluate it as (float)log((double)x), i.e. the correctly rounded
//     binary32 logarithm, so the two sides agree bit-for-bit.
//
// Parity status: the reference needs warp-lang, which is not installed in
// this environment, so it cannot be run to produce golden outputs.  The
// oracle is pinned against (a) the reference's own CPU coverage oracle and
// its seeded 253-case sweep (tests/test_tile_coverage.py:35-279), (b) the
// reference's single-Gaussian compositing oracle
// (tests/test_rasterizer_cuda_contracts.py:451-505) and (c) its
// finite-difference gradient check (:588-607); see tests/test_oracle_*.py.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#include <parallel/algorithm>
#endif

#define OR_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

constexpr int BLOCK_X = 16;
constexpr int BLOCK_Y = 16;
constexpr int NUM_CHANNELS = 3;
constexpr float DET_EPSILON = 1.0e-7f;          // constants.py:38
constexpr float ONE_MINUS_ALPHA_MIN = 1.0e-5f;  // constants.py:39
constexpr float SNUGBOX_PIXEL_PADDING = 1.0f;   // constants.py:40
constexpr float COVERAGE_Q_EPSILON = 1.0e-4f;   // constants.py:41
constexpr int MODE_SNUGBOX = 0;                 // constants.py:42-44
constexpr int MODE_ACCUTILE = 1;
constexpr int MODE_CONIC_RECT = 2;
constexpr float FLT_BIG = 3.402823466e38f;

// constants.py:8-22 (float32 of the listed doubles)
const float SH_C0 = 0.28209479177387814f;
const float SH_C1 = 0.4886025119029199f;
const float SH_C2_0 = 1.0925484305920792f;
const float SH_C2_1 = -1.0925484305920792f;
const float SH_C2_2 = 0.31539156525252005f;
const float SH_C2_3 = -1.0925484305920792f;
const float SH_C2_4 = 0.5462742152960396f;
const float SH_C3_0 = -0.5900435899266435f;
const float SH_C3_1 = 2.890611442640554f;
const float SH_C3_2 = -0.4570457994644658f;
const float SH_C3_3 = 0.3731763325901154f;
const float SH_C3_4 = -0.4570457994644658f;
const float SH_C3_5 = 1.445305721320277f;
const float SH_C3_6 = -0.5900435899266435f;

inline int f2i(float x) {
  // Saturating truncation, NaN -> 0 (cvt.rzi.s32.f32 semantics).
  if (std::isnan(x)) return 0;
  if (x >= 2147483648.0f) return 2147483647;
  if (x <= -2147483648.0f) return (int)(-2147483647 - 1);
  return (int)x;
}
inline int imin(int a, int b) { return a < b ? a : b; }
inline int imax(int a, int b) { return a > b ? a : b; }
inline float fmn(float a, float b) { return a < b ? a : b; }
inline float fmx(float a, float b) { return a > b ? a : b; }
inline float fclamp(float x, float lo, float hi) { return fmn(fmx(x, lo), hi); }

// Correctly rounded binary32 natural log (see header comment).
inline float crlogf(float x) { return (float)std::log((double)x); }

struct Rect { int x0, y0, x1, y1; };

// math_kernels.py:86-87
inline float ndc2pix(float v, int size) {
  return ((v + 1.0f) * (float)size - 1.0f) * 0.5f;
}

// math_kernels.py:136-148
inline Rect tile_rect(float px, float py, int radius, int grid_x, int grid_y) {
  Rect r;
  r.x0 = imin(grid_x, imax(0, f2i((px - (float)radius) / (float)BLOCK_X)));
  r.y0 = imin(grid_y, imax(0, f2i((py - (float)radius) / (float)BLOCK_Y)));
  r.x1 = imin(grid_x, imax(0, f2i((px + (float)radius + (float)(BLOCK_X - 1)) / (float)BLOCK_X)));
  r.y1 = imin(grid_y, imax(0, f2i((py + (float)radius + (float)(BLOCK_Y - 1)) / (float)BLOCK_Y)));
  return r;
}

// math_kernels.py:150-194 (SnugBox clipped to the CUDA 3-sigma rect)
inline Rect snugbox_rect(float px, float py, float cov_aa, float cov_cc, float opacity,
                         int cuda_radius, int grid_x, int grid_y) {
  Rect c = tile_rect(px, py, cuda_radius, grid_x, grid_y);
  float t = 2.0f * crlogf(fmx(255.0f * opacity, 1.0f));
  if (t <= 0.0f) return Rect{0, 0, 0, 0};
  int rx = f2i(std::ceil(std::sqrt(fmx(t * cov_aa, 0.0f)) + SNUGBOX_PIXEL_PADDING));
  int ry = f2i(std::ceil(std::sqrt(fmx(t * cov_cc, 0.0f)) + SNUGBOX_PIXEL_PADDING));
  Rect s;
  s.x0 = imin(grid_x, imax(0, f2i((px - (float)rx) / (float)BLOCK_X)));
  s.y0 = imin(grid_y, imax(0, f2i((py - (float)ry) / (float)BLOCK_Y)));
  s.x1 = imin(grid_x, imax(0, f2i((px + (float)rx + (float)(BLOCK_X - 1)) / (float)BLOCK_X)));
  s.y1 = imin(grid_y, imax(0, f2i((py + (float)ry + (float)(BLOCK_Y - 1)) / (float)BLOCK_Y)));
  return Rect{imax(c.x0, s.x0), imax(c.y0, s.y0), imin(c.x1, s.x1), imin(c.y1, s.y1)};
}

// math_kernels.py:196-204
inline float conic_q(float x, float y, float a, float b, float c) {
  return a * x * x + 2.0f * b * x * y + c * y * y;
}

// math_kernels.py:206-240
inline bool conic_rect_intersects(float px, float py, float a, float b, float c,
                                  float threshold, int tx, int ty) {
  float det = a * c - b * b;
  if (a <= 0.0f || c <= 0.0f || det <= DET_EPSILON) return true;
  float x0 = (float)(tx * BLOCK_X) - px;
  float x1 = (float)(tx * BLOCK_X + BLOCK_X - 1) - px;
  float y0 = (float)(ty * BLOCK_Y) - py;
  float y1 = (float)(ty * BLOCK_Y + BLOCK_Y - 1) - py;
  if (x0 <= 0.0f && x1 >= 0.0f && y0 <= 0.0f && y1 >= 0.0f) return true;
  float q_min = FLT_BIG;
  float y = fclamp(-b * x0 / c, y0, y1);
  q_min = fmn(q_min, conic_q(x0, y, a, b, c));
  y = fclamp(-b * x1 / c, y0, y1);
  q_min = fmn(q_min, conic_q(x1, y, a, b, c));
  float x = fclamp(-b * y0 / a, x0, x1);
  q_min = fmn(q_min, conic_q(x, y0, a, b, c));
  x = fclamp(-b * y1 / a, x0, x1);
  q_min = fmn(q_min, conic_q(x, y1, a, b, c));
  return q_min <= threshold + COVERAGE_Q_EPSILON;
}

// math_kernels.py:242-303 (AccuTile: tile interval of one band)
inline void band_interval(float pu, float pv, float cuu, float cuv, float cvv, float threshold,
                          int tile_v, int block_u, int block_v, int rect_u_min, int rect_u_max,
                          int* lo, int* hi) {
  float det = cuu * cvv - cuv * cuv;
  if (cuu <= 0.0f || cvv <= 0.0f || det <= DET_EPSILON) {
    *lo = rect_u_min;
    *hi = rect_u_max;
    return;
  }
  float ts = threshold + COVERAGE_Q_EPSILON;
  float v0 = (float)(tile_v * block_v) - pv;
  float v1 = (float)(tile_v * block_v + block_v - 1) - pv;
  float u_min = FLT_BIG, u_max = -FLT_BIG;
  bool found = false;
  float disc = cuu * ts - det * v0 * v0;
  if (disc >= -COVERAGE_Q_EPSILON) {
    float half = std::sqrt(fmx(disc, 0.0f)) / cuu;
    float center = -cuv * v0 / cuu;
    u_min = fmn(u_min, center - half);
    u_max = fmx(u_max, center + half);
    found = true;
  }
  disc = cuu * ts - det * v1 * v1;
  if (disc >= -COVERAGE_Q_EPSILON) {
    float half = std::sqrt(fmx(disc, 0.0f)) / cuu;
    float center = -cuv * v1 / cuu;
    u_min = fmn(u_min, center - half);
    u_max = fmx(u_max, center + half);
    found = true;
  }
  float extent_u = std::sqrt(fmx(ts * cvv / det, 0.0f));
  float v_at_min_u = cuv * extent_u / cvv;
  if (v_at_min_u >= v0 - COVERAGE_Q_EPSILON && v_at_min_u <= v1 + COVERAGE_Q_EPSILON) {
    u_min = fmn(u_min, -extent_u);
    u_max = fmx(u_max, -extent_u);
    found = true;
  }
  float v_at_max_u = -cuv * extent_u / cvv;
  if (v_at_max_u >= v0 - COVERAGE_Q_EPSILON && v_at_max_u <= v1 + COVERAGE_Q_EPSILON) {
    u_min = fmn(u_min, extent_u);
    u_max = fmx(u_max, extent_u);
    found = true;
  }
  if (!found) {
    *lo = rect_u_min;
    *hi = rect_u_min;
    return;
  }
  int tmin = f2i(std::floor((pu + u_min) / (float)block_u));
  int tmax = f2i(std::floor((pu + u_max) / (float)block_u)) + 1;
  *lo = imax(rect_u_min, imin(rect_u_max, tmin));
  *hi = imax(rect_u_min, imin(rect_u_max, tmax));
}

// math_kernels.py:305-390 (tile count) and binning_kernels.py:126-216 (emit).
// emit==nullptr: count only.  Otherwise append tile ids in the reference's
// emission order.
inline int cover_tiles(float px, float py, float cov_aa, float cov_cc, float ca, float cb,
                       float cc, float opacity, int cuda_radius, int grid_x, int grid_y,
                       int mode, std::vector<int>* emit) {
  Rect r = snugbox_rect(px, py, cov_aa, cov_cc, opacity, cuda_radius, grid_x, grid_y);
  int span_x = r.x1 - r.x0;
  int span_y = r.y1 - r.y0;
  int area = span_x * span_y;
  if (area <= 1 || mode == MODE_SNUGBOX) {
    if (emit) {
      for (int ty = r.y0; ty < r.y1; ++ty)
        for (int tx = r.x0; tx < r.x1; ++tx) emit->push_back(ty * grid_x + tx);
    }
    return area;
  }
  float threshold = 2.0f * crlogf(fmx(255.0f * opacity, 1.0f));
  int count = 0;
  // conic_rect: per-tile test up to 64 tiles, AccuTile above (the recount
  // binning applies, binning_kernels.py:56-124).
  if (mode == MODE_CONIC_RECT && area <= 64) {
    for (int ty = r.y0; ty < r.y1; ++ty)
      for (int tx = r.x0; tx < r.x1; ++tx)
        if (conic_rect_intersects(px, py, ca, cb, cc, threshold, tx, ty)) {
          ++count;
          if (emit) emit->push_back(ty * grid_x + tx);
        }
    return count;
  }
  if (span_y <= span_x) {
    for (int ty = r.y0; ty < r.y1; ++ty) {
      int lo, hi;
      band_interval(px, py, ca, cb, cc, threshold, ty, BLOCK_X, BLOCK_Y, r.x0, r.x1, &lo, &hi);
      count += imax(0, hi - lo);
      if (emit)
        for (int tx = lo; tx < hi; ++tx) emit->push_back(ty * grid_x + tx);
    }
  } else {
    for (int tx = r.x0; tx < r.x1; ++tx) {
      int lo, hi;
      band_interval(py, px, cc, cb, ca, threshold, tx, BLOCK_Y, BLOCK_X, r.y0, r.y1, &lo, &hi);
      count += imax(0, hi - lo);
      if (emit)
        for (int ty = lo; ty < hi; ++ty) emit->push_back(ty * grid_x + tx);
    }
  }
  return count;
}

struct Mat { const float* v; };

inline float dot_row_view_z(const float* v, const float* p) {
  return v[2] * p[0] + v[6] * p[1] + v[10] * p[2] + v[14];
}

// Fills the common screen-space outputs once cov2d (a,b,c) is known.
// preprocess_kernels.py:221-269 (fused path) / :439-476 (cov3D_precomp path).
// Returns true when the Gaussian survives.
struct PreOut {
  float* depths; int* radii; float* proj_2d; float* conic_2d; float* conic_2d_inv;
  int* tiles_touched; float* conic_opacity;
};

inline void finish_screen_space(int idx, float cov_a, float cov_b, float cov_c, bool strict_det,
                                float p_proj_x, float p_proj_y, float depth, float opacity,
                                int W, int H, int grid_x, int grid_y, int mode, const PreOut& o) {
  float det = cov_a * cov_c - cov_b * cov_b;
  if (strict_det ? (std::fabs(det) < DET_EPSILON) : (std::fabs(det) <= DET_EPSILON)) return;
  float det_inv = 1.0f / det;
  float con0 = cov_c * det_inv, con1 = -cov_b * det_inv, con2 = cov_a * det_inv;
  float mid = 0.5f * (cov_a + cov_c);
  float root = std::sqrt(fmx(0.1f, mid * mid - det));
  float l1 = mid + root, l2 = mid - root;
  int radius = f2i(std::ceil(3.0f * std::sqrt(fmx(l1, l2))));
  float px = ndc2pix(p_proj_x, W);
  float py = ndc2pix(p_proj_y, H);
  Rect cr = tile_rect(px, py, radius, grid_x, grid_y);
  if ((cr.x1 - cr.x0) * (cr.y1 - cr.y0) == 0) return;
  o.depths[idx] = depth;
  o.radii[idx] = radius;
  o.proj_2d[idx * 2 + 0] = px;
  o.proj_2d[idx * 2 + 1] = py;
  o.conic_2d[idx * 3 + 0] = con0;
  o.conic_2d[idx * 3 + 1] = con1;
  o.conic_2d[idx * 3 + 2] = con2;
  o.conic_2d_inv[idx * 3 + 0] = cov_a;
  o.conic_2d_inv[idx * 3 + 1] = cov_b;
  o.conic_2d_inv[idx * 3 + 2] = cov_c;
  o.conic_opacity[idx * 4 + 0] = con0;
  o.conic_opacity[idx * 4 + 1] = con1;
  o.conic_opacity[idx * 4 + 2] = con2;
  o.conic_opacity[idx * 4 + 3] = opacity;
  o.tiles_touched[idx] = cover_tiles(px, py, cov_a, cov_c, con0, con1, con2, opacity, radius,
                                     grid_x, grid_y, mode, nullptr);
}

// R(q) * diag(s) rows as used by every cov3d site (preprocess_kernels.py:156-174)
struct MRows { float m00, m01, m02, m10, m11, m12, m20, m21, m22; float r00, r01, r02, r10, r11, r12, r20, r21, r22; };
inline MRows make_m(const float* scale, const float* q, float mod) {
  float s0 = scale[0] * mod, s1 = scale[1] * mod, s2 = scale[2] * mod;
  float rr = q[0], xq = q[1], yq = q[2], zq = q[3];
  MRows m;
  m.r00 = 1.0f - 2.0f * (yq * yq + zq * zq);
  m.r01 = 2.0f * (xq * yq + rr * zq);
  m.r02 = 2.0f * (xq * zq - rr * yq);
  m.r10 = 2.0f * (xq * yq - rr * zq);
  m.r11 = 1.0f - 2.0f * (xq * xq + zq * zq);
  m.r12 = 2.0f * (yq * zq + rr * xq);
  m.r20 = 2.0f * (xq * zq + rr * yq);
  m.r21 = 2.0f * (yq * zq - rr * xq);
  m.r22 = 1.0f - 2.0f * (xq * xq + yq * yq);
  m.m00 = s0 * m.r00; m.m01 = s0 * m.r01; m.m02 = s0 * m.r02;
  m.m10 = s1 * m.r10; m.m11 = s1 * m.r11; m.m12 = s1 * m.r12;
  m.m20 = s2 * m.r20; m.m21 = s2 * m.r21; m.m22 = s2 * m.r22;
  return m;
}

}  // namespace

// ---------------------------------------------------------------------------
// Single-Gaussian coverage helpers (tests pin these against the reference's
// coverage oracle, tests/test_tile_coverage.py:35-163).
// ---------------------------------------------------------------------------
OR_EXPORT int or_count_tiles(float px, float py, float cov_aa, float cov_cc, float ca, float cb,
                             float cc, float opacity, int cuda_radius, int grid_x, int grid_y,
                             int mode) {
  return cover_tiles(px, py, cov_aa, cov_cc, ca, cb, cc, opacity, cuda_radius, grid_x, grid_y,
                     mode, nullptr);
}

OR_EXPORT int or_emit_tiles(float px, float py, float cov_aa, float cov_cc, float ca, float cb,
                            float cc, float opacity, int cuda_radius, int grid_x, int grid_y,
                            int mode, int* out, int cap) {
  std::vector<int> e;
  cover_tiles(px, py, cov_aa, cov_cc, ca, cb, cc, opacity, cuda_radius, grid_x, grid_y, mode, &e);
  int n = (int)e.size();
  for (int i = 0; i < n && i < cap; ++i) out[i] = e[i];
  return n;
}

OR_EXPORT float or_threshold_log(float x) { return crlogf(x); }

OR_EXPORT void or_threshold_log_batch(const float* x, float* out, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) out[i] = crlogf(x[i]);
}

// ---------------------------------------------------------------------------
// Preprocess forward.  Fused scale/rotation path:
// preprocess_kernels.py:83-269 + SH colour preprocess_kernels.py:272-342.
// cov3D_precomp path: preprocess_kernels.py:630-672 (visibility) + :345-476.
// sh == nullptr -> colours are not evaluated (colors_precomp path).
// ---------------------------------------------------------------------------
OR_EXPORT void or_preprocess_fwd(
    int P, const float* means, const float* scales, const float* rotations, float scale_modifier,
    const float* cov3d_precomp, const float* opacities, const float* view, const float* proj,
    float tanfovx, float tanfovy, float focal_x, float focal_y, int W, int H, int mode,
    const float* sh, int degree, int coeff_count, const float* campos,
    // outputs
    float* cov3d, int* visible, float* depths, int* radii, float* proj_2d, float* conic_2d,
    float* conic_2d_inv, int* tiles_touched, float* conic_opacity, float* rgb, int* clamped) {
  const int grid_x = (W + BLOCK_X - 1) / BLOCK_X;
  const int grid_y = (H + BLOCK_Y - 1) / BLOCK_Y;
  PreOut o{depths, radii, proj_2d, conic_2d, conic_2d_inv, tiles_touched, conic_opacity};
#pragma omp parallel for schedule(static)
  for (int idx = 0; idx < P; ++idx) {
    for (int k = 0; k < 6; ++k) cov3d[idx * 6 + k] = cov3d_precomp ? cov3d_precomp[idx * 6 + k] : 0.0f;
    depths[idx] = 0.0f;
    radii[idx] = 0;
    proj_2d[idx * 2] = proj_2d[idx * 2 + 1] = 0.0f;
    for (int k = 0; k < 3; ++k) conic_2d[idx * 3 + k] = conic_2d_inv[idx * 3 + k] = 0.0f;
    tiles_touched[idx] = 0;
    for (int k = 0; k < 4; ++k) conic_opacity[idx * 4 + k] = 0.0f;
    const float* p = means + idx * 3;
    const float* v = view;
    const float* pr = proj;
    float p_view_z = dot_row_view_z(v, p);
    if (!cov3d_precomp) {
      // ---- fused scale/rotation path ----
      if (p_view_z <= 0.2f) {
        visible[idx] = 0;
      } else {
        visible[idx] = 1;
        float hom_x = pr[0] * p[0] + pr[4] * p[1] + pr[8] * p[2] + pr[12];
        float hom_y = pr[1] * p[0] + pr[5] * p[1] + pr[9] * p[2] + pr[13];
        float hom_w = pr[3] * p[0] + pr[7] * p[1] + pr[11] * p[2] + pr[15];
        float inv_w = 1.0f / (hom_w + 1.0e-7f);
        float ppx = hom_x * inv_w, ppy = hom_y * inv_w;
        MRows m = make_m(scales + idx * 3, rotations + idx * 4, scale_modifier);
        float* c3 = cov3d + idx * 6;
        c3[0] = m.m00 * m.m00 + m.m10 * m.m10 + m.m20 * m.m20;
        c3[1] = m.m00 * m.m01 + m.m10 * m.m11 + m.m20 * m.m21;
        c3[2] = m.m00 * m.m02 + m.m10 * m.m12 + m.m20 * m.m22;
        c3[3] = m.m01 * m.m01 + m.m11 * m.m11 + m.m21 * m.m21;
        c3[4] = m.m01 * m.m02 + m.m11 * m.m12 + m.m21 * m.m22;
        c3[5] = m.m02 * m.m02 + m.m12 * m.m12 + m.m22 * m.m22;
        float vx = v[0] * p[0] + v[4] * p[1] + v[8] * p[2] + v[12];
        float vy = v[1] * p[0] + v[5] * p[1] + v[9] * p[2] + v[13];
        float vz = p_view_z;
        float limx = 1.3f * tanfovx, limy = 1.3f * tanfovy;
        float txtz = vx / vz, tytz = vy / vz;
        vx = fclamp(txtz, -limx, limx) * vz;
        vy = fclamp(tytz, -limy, limy) * vz;
        float a_j = focal_x / vz, b_j = focal_y / vz;
        float c_j = -(focal_x * vx) / (vz * vz);
        float d_j = -(focal_y * vy) / (vz * vz);
        float t00 = v[0] * a_j + v[2] * c_j;
        float t10 = v[4] * a_j + v[6] * c_j;
        float t20 = v[8] * a_j + v[10] * c_j;
        float t01 = v[1] * b_j + v[2] * d_j;
        float t11 = v[5] * b_j + v[6] * d_j;
        float t21 = v[9] * b_j + v[10] * d_j;
        float a00 = m.m00 * t00 + m.m01 * t10 + m.m02 * t20;
        float a10 = m.m10 * t00 + m.m11 * t10 + m.m12 * t20;
        float a20 = m.m20 * t00 + m.m21 * t10 + m.m22 * t20;
        float a01 = m.m00 * t01 + m.m01 * t11 + m.m02 * t21;
        float a11 = m.m10 * t01 + m.m11 * t11 + m.m12 * t21;
        float a21 = m.m20 * t01 + m.m21 * t11 + m.m22 * t21;
        float cov_a = a00 * a00 + a10 * a10 + a20 * a20 + 0.3f;
        float cov_b = a00 * a01 + a10 * a11 + a20 * a21;
        float cov_c = a01 * a01 + a11 * a11 + a21 * a21 + 0.3f;
        finish_screen_space(idx, cov_a, cov_b, cov_c, false, ppx, ppy, p_view_z, opacities[idx], W,
                            H, grid_x, grid_y, mode, o);
      }
    } else {
      // ---- cov3D_precomp path: visibility (preprocess_kernels.py:630-672) ----
      bool vis = false;
      float ppx = 0.0f, ppy = 0.0f;
      if (p_view_z > 0.2f) {
        float hom_x = pr[0] * p[0] + pr[4] * p[1] + pr[8] * p[2] + pr[12];
        float hom_y = pr[1] * p[0] + pr[5] * p[1] + pr[9] * p[2] + pr[13];
        float hom_w = pr[3] * p[0] + pr[7] * p[1] + pr[11] * p[2] + pr[15];
        float inv_w = 1.0f / (hom_w + 1.0e-7f);
        ppx = hom_x * inv_w;
        ppy = hom_y * inv_w;
        const float* c3 = cov3d_precomp + idx * 6;
        // math_kernels.py:104-115
        float row0 = std::fabs(c3[0]) + std::fabs(c3[1]) + std::fabs(c3[2]);
        float row1 = std::fabs(c3[1]) + std::fabs(c3[3]) + std::fabs(c3[4]);
        float row2 = std::fabs(c3[2]) + std::fabs(c3[4]) + std::fabs(c3[5]);
        float lam = fmx(row0, fmx(row1, row2));
        // math_kernels.py:117-134 (focal recomputed in float inside the kernel)
        float limx = 1.3f * tanfovx, limy = 1.3f * tanfovy;
        float fx = (float)W / (2.0f * tanfovx);
        float fy = (float)H / (2.0f * tanfovy);
        float row0n = (fx / p_view_z) * std::sqrt(1.0f + limx * limx);
        float row1n = (fy / p_view_z) * std::sqrt(1.0f + limy * limy);
        float jf = row0n * row0n + row1n * row1n;
        float lu = lam * jf + 0.3f;
        int radius_upper = f2i(std::ceil(3.0f * std::sqrt(fmx(lu, 0.0f))));
        // math_kernels.py:392-406
        float qx = ndc2pix(ppx, W), qy = ndc2pix(ppy, H);
        Rect rr = tile_rect(qx, qy, radius_upper, grid_x, grid_y);
        vis = (rr.x1 - rr.x0) * (rr.y1 - rr.y0) != 0;
      }
      visible[idx] = vis ? 1 : 0;
      if (vis) {
        // preprocess_kernels.py:385-476
        float x = v[0] * p[0] + v[4] * p[1] + v[8] * p[2] + v[12];
        float y = v[1] * p[0] + v[5] * p[1] + v[9] * p[2] + v[13];
        float z = v[2] * p[0] + v[6] * p[1] + v[10] * p[2] + v[14];
        float limx = 1.3f * tanfovx, limy = 1.3f * tanfovy;
        float txtz = x / z, tytz = y / z;
        x = fclamp(txtz, -limx, limx) * z;
        y = fclamp(tytz, -limy, limy) * z;
        float a = focal_x / z, b = focal_y / z;
        float c = -(focal_x * x) / (z * z);
        float d = -(focal_y * y) / (z * z);
        float t00 = v[0] * a + v[2] * c;
        float t10 = v[4] * a + v[6] * c;
        float t20 = v[8] * a + v[10] * c;
        float t01 = v[1] * b + v[2] * d;
        float t11 = v[5] * b + v[6] * d;
        float t21 = v[9] * b + v[10] * d;
        const float* c3 = cov3d_precomp + idx * 6;
        float v00 = c3[0], v01 = c3[1], v02 = c3[2], v11 = c3[3], v12 = c3[4], v22 = c3[5];
        float vt0x = v00 * t00 + v01 * t10 + v02 * t20;
        float vt0y = v01 * t00 + v11 * t10 + v12 * t20;
        float vt0z = v02 * t00 + v12 * t10 + v22 * t20;
        float vt1x = v00 * t01 + v01 * t11 + v02 * t21;
        float vt1y = v01 * t01 + v11 * t11 + v12 * t21;
        float vt1z = v02 * t01 + v12 * t11 + v22 * t21;
        float cov_a = t00 * vt0x + t10 * vt0y + t20 * vt0z + 0.3f;
        float cov_b = t00 * vt1x + t10 * vt1y + t20 * vt1z;
        float cov_c = t01 * vt1x + t11 * vt1y + t21 * vt1z + 0.3f;
        finish_screen_space(idx, cov_a, cov_b, cov_c, true, ppx, ppy, p_view_z, opacities[idx], W,
                            H, grid_x, grid_y, mode, o);
      }
    }

    // ---- SH -> RGB (preprocess_kernels.py:272-342), evaluated for every Gaussian ----
    if (sh) {
      const float* sp = sh + (size_t)idx * coeff_count * 3;
      float dx = p[0] - campos[0], dy = p[1] - campos[1], dz = p[2] - campos[2];
      float len_sq = dx * dx + dy * dy + dz * dz;
      float inv_len = 1.0f / std::sqrt(fmx(len_sq, 1.0e-20f));
      float x = dx * inv_len, y = dy * inv_len, z = dz * inv_len;
      float col[3];
      for (int ch = 0; ch < 3; ++ch) col[ch] = SH_C0 * sp[ch];
      if (degree > 0 && coeff_count > 3) {
        float b1 = -SH_C1 * y, b2 = SH_C1 * z, b3 = -SH_C1 * x;
        for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + b1 * sp[3 + ch];
        for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + b2 * sp[6 + ch];
        for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + b3 * sp[9 + ch];
        if (degree > 1 && coeff_count > 8) {
          float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
          float w4 = SH_C2_0 * xy, w5 = SH_C2_1 * yz, w6 = SH_C2_2 * (2.0f * zz - xx - yy);
          float w7 = SH_C2_3 * xz, w8 = SH_C2_4 * (xx - yy);
          for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w4 * sp[12 + ch];
          for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w5 * sp[15 + ch];
          for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w6 * sp[18 + ch];
          for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w7 * sp[21 + ch];
          for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w8 * sp[24 + ch];
          if (degree > 2 && coeff_count > 15) {
            float w9 = SH_C3_0 * y * (3.0f * xx - yy);
            float w10 = SH_C3_1 * xy * z;
            float w11 = SH_C3_2 * y * (4.0f * zz - xx - yy);
            float w12 = SH_C3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
            float w13 = SH_C3_4 * x * (4.0f * zz - xx - yy);
            float w14 = SH_C3_5 * z * (xx - yy);
            float w15 = SH_C3_6 * x * (xx - 3.0f * yy);
            const float w[7] = {w9, w10, w11, w12, w13, w14, w15};
            for (int k = 0; k < 7; ++k)
              for (int ch = 0; ch < 3; ++ch) col[ch] = col[ch] + w[k] * sp[(9 + k) * 3 + ch];
          }
        }
      }
      for (int ch = 0; ch < 3; ++ch) {
        float cval = col[ch] + 0.5f;
        int cl = 0;
        if (cval < 0.0f) { cval = 0.0f; cl = 1; }
        rgb[idx * 3 + ch] = cval;
        clamped[idx * 3 + ch] = cl;
      }
    }
  }
}

// mark_visible (preprocess_kernels.py:603-627): p_view_z > 0.2
OR_EXPORT void or_mark_visible(int P, const float* means, const float* view, unsigned char* out) {
  for (int i = 0; i < P; ++i) out[i] = dot_row_view_z(view, means + i * 3) > 0.2f ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Binning (binning_ops.py:84-431).  Canonical order of the sorted pair list:
// ascending (tile id, depth float bits, point index).  Both reference sort
// modes produce it (stable depth sort + stable tile sort, or stable 64-bit
// (tile<<32|depth bits) sort over index-ordered emission).
// Returns num_rendered; point_list must hold it (call with cap=0 to size).
// ranges: (tiles, 2) int32, empty tiles (0,0).
// ---------------------------------------------------------------------------
OR_EXPORT long long or_binning(int P, const float* xy, const int* radii, const float* conic_opacity,
                               const float* conic_2d_inv, const float* depths,
                               const int* tiles_touched, int W, int H, int mode,
                               int* point_list, long long cap, int* ranges, int* tile_keys) {
  const int grid_x = (W + BLOCK_X - 1) / BLOCK_X;
  const int grid_y = (H + BLOCK_Y - 1) / BLOCK_Y;
  const int T = grid_x * grid_y;
  // pair slots of each Gaussian: exclusive prefix sum of tiles_touched
  std::vector<long long> offset((size_t)P + 1, 0);
  for (int i = 0; i < P; ++i) offset[i + 1] = offset[i] + tiles_touched[i];
  const long long total = offset[P];
  if (cap < total) return total;
  struct Pair { uint32_t tile; uint32_t depth; uint32_t idx; };
  std::vector<Pair> pairs((size_t)total);
  int mismatch = 0;
#pragma omp parallel reduction(| : mismatch)
  {
    std::vector<int> e;
#pragma omp for schedule(dynamic, 4096)
    for (int i = 0; i < P; ++i) {
      if (radii[i] <= 0) continue;
      e.clear();
      const float* co = conic_opacity + i * 4;
      const float* cv = conic_2d_inv + i * 3;
      cover_tiles(xy[i * 2], xy[i * 2 + 1], cv[0], cv[2], co[0], co[1], co[2], co[3], radii[i],
                  grid_x, grid_y, mode, &e);
      if ((long long)e.size() != tiles_touched[i]) {
        mismatch = 1;
        continue;
      }
      uint32_t db;
      std::memcpy(&db, &depths[i], 4);
      for (size_t k = 0; k < e.size(); ++k) pairs[(size_t)offset[i] + k] = Pair{(uint32_t)e[k], db, (uint32_t)i};
    }
  }
  if (mismatch) return -1;  // count/emit disagreement
  // (tile, depth bits, index) is a total order on the pairs: any correct sort gives the same list
  __gnu_parallel::sort(pairs.begin(), pairs.end(), [](const Pair& a, const Pair& b) {
    if (a.tile != b.tile) return a.tile < b.tile;
    if (a.depth != b.depth) return a.depth < b.depth;
    return a.idx < b.idx;
  });
  for (int t = 0; t < 2 * T; ++t) ranges[t] = 0;
  for (long long k = 0; k < total; ++k) {
    point_list[k] = (int)pairs[k].idx;
    if (tile_keys) tile_keys[k] = (int)pairs[k].tile;
    int t = (int)pairs[k].tile;
    if (k == 0 || pairs[k - 1].tile != pairs[k].tile) ranges[2 * t] = (int)k;
    if (k == total - 1 || pairs[k + 1].tile != pairs[k].tile) ranges[2 * t + 1] = (int)(k + 1);
  }
  return total;
}

// Relative distance of a pixel's thresholded decisions from their thresholds
// (test instrumentation, not part of the reference's arithmetic): the sign
// test of the exponent against the size of its terms, alpha >= 1/255 and
// T*(1-alpha) < 1e-4.  An implementation whose exp or exponent rounding
// differs by a relative d can decide a pair differently only where this is
// below about d.
inline float power_scale(float a, float b, float c, float dx, float dy) {
  return 0.5f * (std::fabs(a) * dx * dx + std::fabs(c) * dy * dy) + std::fabs(b * dx * dy);
}
inline float power_margin(float power, float a, float b, float c, float dx, float dy) {
  const float scale = power_scale(a, b, c, dx, dy);
  return scale > 0.0f ? std::fabs(power) / scale : 1.0f;
}
inline float alpha_margin(float alpha) { return std::fabs(alpha - 1.0f / 255.0f) * 255.0f; }
inline float trans_margin(float test_T) { return std::fabs(test_T - 0.0001f) * 10000.0f; }

// ---------------------------------------------------------------------------
// Render forward (render_kernels.py:15-147).  Integer pixel coordinates,
// front-to-back, stop when T*(1-alpha) < 1e-4 without adding that pair.
// margin (optional, per pixel): the smallest decision margin of the pairs the
// pixel evaluates (see power_margin); cond (optional, per pixel): the largest
// power_scale of the pairs it blends -- the absolute size of the terms whose
// sum is the exponent, so rounding differences in the exponent are of order
// eps * cond.
// ---------------------------------------------------------------------------
OR_EXPORT void or_render_fwd(int W, int H, const int* ranges, const int* point_list,
                             const float* xy, const float* features, const float* depths,
                             const float* conic_opacity, const float* bg, int compute_depth,
                             float* out_color, float* out_depth, float* out_alpha, int* n_contrib,
                             float* margin, float* cond) {
  const int grid_x = (W + BLOCK_X - 1) / BLOCK_X;
  const int grid_y = (H + BLOCK_Y - 1) / BLOCK_Y;
  const long long npix = (long long)W * H;
#pragma omp parallel for schedule(dynamic, 4)
  for (int tile = 0; tile < grid_x * grid_y; ++tile) {
    int tx = tile % grid_x, ty = tile / grid_x;
    int start = ranges[2 * tile], end = ranges[2 * tile + 1];
    for (int local = 0; local < BLOCK_X * BLOCK_Y; ++local) {
      int pxi = tx * BLOCK_X + local % BLOCK_X;
      int pyi = ty * BLOCK_Y + local / BLOCK_X;
      if (pxi >= W || pyi >= H) continue;
      long long pix = (long long)pyi * W + pxi;
      float T = 1.0f, c0 = 0, c1 = 0, c2 = 0, wsum = 0, dacc = 0;
      int contributor = 0, last = 0;
      float fx = (float)pxi, fy = (float)pyi;
      float m = 1.0f, cd = 0.0f;
      for (int k = start; k < end; ++k) {
        contributor = contributor + 1;
        int id = point_list[k];
        const float* co = conic_opacity + id * 4;
        float d_x = xy[id * 2] - fx;
        float d_y = xy[id * 2 + 1] - fy;
        float power = -0.5f * (co[0] * d_x * d_x + co[2] * d_y * d_y) - co[1] * d_x * d_y;
        if (margin) m = fmn(m, power_margin(power, co[0], co[1], co[2], d_x, d_y));
        if (power <= 0.0f) {
          float alpha = fmn(0.99f, co[3] * std::exp(power));
          if (margin) m = fmn(m, alpha_margin(alpha));
          if (alpha >= (1.0f / 255.0f)) {
            float test_T = T * (1.0f - alpha);
            if (margin) m = fmn(m, trans_margin(test_T));
            if (test_T < 0.0001f) break;
            float contribution = alpha * T;
            if (cond) cd = fmx(cd, power_scale(co[0], co[1], co[2], d_x, d_y));
            c0 = c0 + features[id * 3 + 0] * contribution;
            c1 = c1 + features[id * 3 + 1] * contribution;
            c2 = c2 + features[id * 3 + 2] * contribution;
            wsum = wsum + contribution;
            if (compute_depth) dacc = dacc + depths[id] * contribution;
            T = test_T;
            last = contributor;
          }
        }
      }
      n_contrib[pix] = last;
      if (margin) margin[pix] = m;
      if (cond) cond[pix] = cd;
      out_color[pix] = c0 + T * bg[0];
      out_color[npix + pix] = c1 + T * bg[1];
      out_color[2 * npix + pix] = c2 + T * bg[2];
      out_alpha[pix] = wsum;
      out_depth[pix] = dacc;
    }
  }
}

// ---------------------------------------------------------------------------
// Flow auxiliary outputs of the flow render (flow_kernels.py:14-180): the
// same front-to-back loop as or_render_fwd; the first `top_k` Gaussians that
// contribute to a pixel are recorded in order with their compositing weight
// (alpha * T) and the offset (dx, dy) = centre - pixel.  Slots that stay
// empty keep -1 / 0 / 0 (flow_ops.py:119-125).
// ---------------------------------------------------------------------------
OR_EXPORT void or_render_flow_aux(int W, int H, const int* ranges, const int* point_list, const float* xy,
                                  const float* conic_opacity, int top_k, int* gs_per_pixel,
                                  float* weight_per_gs_pixel, float* x_mu) {
  const int grid_x = (W + BLOCK_X - 1) / BLOCK_X;
  const int grid_y = (H + BLOCK_Y - 1) / BLOCK_Y;
  const long long npix = (long long)W * H;
  for (long long i = 0; i < (long long)top_k * npix; ++i) {
    gs_per_pixel[i] = -1;
    weight_per_gs_pixel[i] = 0.0f;
    x_mu[i] = 0.0f;
    x_mu[(long long)top_k * npix + i] = 0.0f;
  }
#pragma omp parallel for schedule(dynamic, 4)
  for (int tile = 0; tile < grid_x * grid_y; ++tile) {
    int tx = tile % grid_x, ty = tile / grid_x;
    int start = ranges[2 * tile], end = ranges[2 * tile + 1];
    for (int local = 0; local < BLOCK_X * BLOCK_Y; ++local) {
      int pxi = tx * BLOCK_X + local % BLOCK_X;
      int pyi = ty * BLOCK_Y + local / BLOCK_X;
      if (pxi >= W || pyi >= H) continue;
      long long pix = (long long)pyi * W + pxi;
      float T = 1.0f;
      int n_success = 0;
      float fx = (float)pxi, fy = (float)pyi;
      for (int k = start; k < end; ++k) {
        int id = point_list[k];
        const float* co = conic_opacity + id * 4;
        float d_x = xy[id * 2] - fx;
        float d_y = xy[id * 2 + 1] - fy;
        float power = -0.5f * (co[0] * d_x * d_x + co[2] * d_y * d_y) - co[1] * d_x * d_y;
        if (power <= 0.0f) {
          float alpha = fmn(0.99f, co[3] * std::exp(power));
          if (alpha >= (1.0f / 255.0f)) {
            float test_T = T * (1.0f - alpha);
            if (test_T < 0.0001f) break;
            float contribution = alpha * T;
            if (n_success < top_k) {
              long long a = (long long)n_success * npix + pix;
              gs_per_pixel[a] = id;
              weight_per_gs_pixel[a] = contribution;
              x_mu[a] = d_x;
              x_mu[(long long)top_k * npix + a] = d_y;
            }
            n_success = n_success + 1;
            T = test_T;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Render backward (backward_kernels.py:538-707).  Per-pixel back-to-front
// recurrence.  Per-Gaussian gradients are reduced in double, tile by tile in
// tile order, so the oracle is deterministic.  grad_abs (optional, 10 per G)
// receives the sum of |term| of every accumulated contribution, for
// condition-aware comparison against float atomics.  Test instrumentation
// (optional): margin, per pixel, the smallest decision margin of the pairs
// the backward re-evaluates; flagged_abs (10 per G), the sum of |term| of the
// contributions from pixels whose margin is below flag_eps -- the part of a
// gradient that another exp implementation may decide differently; cond_abs
// (10 per G), the sum of |term| * power_scale over the taken pairs -- each
// term's sensitivity to rounding in its exponent, which is of order eps times
// the size of the exponent's terms.
// Output layout per Gaussian: grad_xy[2], grad_depth[1], grad_co[4], grad_rgb[3].
// ---------------------------------------------------------------------------
OR_EXPORT void or_render_bwd(int W, int H, int P, const int* ranges, const int* point_list,
                             const float* xy, const float* features, const float* depths,
                             const float* conic_opacity, const float* bg, const float* out_alpha,
                             const int* n_contrib, const float* grad_color,
                             const float* grad_depth, const float* grad_alpha, int compute_depth,
                             float* grad_xy, float* grad_depths, float* grad_co, float* grad_rgb,
                             double* grad_abs, float* margin, float flag_eps, double* flagged_abs,
                             double* cond_abs) {
  const int grid_x = (W + BLOCK_X - 1) / BLOCK_X;
  const int grid_y = (H + BLOCK_Y - 1) / BLOCK_Y;
  const int ntile = grid_x * grid_y;
  const long long npix = (long long)W * H;
  const float ddelx_dx = 0.5f * (float)W;
  const float ddely_dy = 0.5f * (float)H;
  // per tile and list position: 10 sums, then (if asked for) 10 sums of |term| and 10 sums of
  // |term| from flagged pixels
  const int OFF_ABS = 10, OFF_COND = grad_abs ? 20 : 10;
  const int OFF_FLAG = OFF_COND + (cond_abs ? 10 : 0);
  const int ACC = OFF_FLAG + (flagged_abs ? 10 : 0);
  // One slot of ACC doubles per entry of the point list (tile lists are
  // contiguous in it), in a grow-only buffer kept across calls; each tile's
  // slots are zeroed by the thread that fills them.
  long long R = 0;
  for (int tile = 0; tile < ntile; ++tile) R = std::max<long long>(R, ranges[2 * tile + 1]);
  static std::vector<double> g_acc;
  if (g_acc.size() < (size_t)R * ACC) g_acc.resize((size_t)R * ACC);
  double* const acc_all = g_acc.data();
#pragma omp parallel for schedule(dynamic, 4)
  for (int tile = 0; tile < ntile; ++tile) {
    int tx = tile % grid_x, ty = tile / grid_x;
    int start = ranges[2 * tile], end = ranges[2 * tile + 1];
    int n = end - start;
    if (n <= 0) continue;
    double* const acc = acc_all + (size_t)start * ACC;
    std::fill(acc, acc + (size_t)n * ACC, 0.0);
    for (int local = 0; local < BLOCK_X * BLOCK_Y; ++local) {
      int pxi = tx * BLOCK_X + local % BLOCK_X;
      int pyi = ty * BLOCK_Y + local / BLOCK_X;
      if (pxi >= W || pyi >= H) continue;
      long long pix = (long long)pyi * W + pxi;
      int lc = n_contrib[pix];
      // with flagged_abs: this pixel's decision margin first (same decisions as below)
      bool flagged = false;
      if (flagged_abs) {
        float pm = 1.0f;
        for (int pos = lc - 1; pos >= 0; --pos) {
          int id = point_list[start + pos];
          const float* co = conic_opacity + id * 4;
          float d_x = xy[id * 2] - (float)pxi;
          float d_y = xy[id * 2 + 1] - (float)pyi;
          float power = -0.5f * (co[0] * d_x * d_x + co[2] * d_y * d_y) - co[1] * d_x * d_y;
          pm = fmn(pm, power_margin(power, co[0], co[1], co[2], d_x, d_y));
          if (power > 0.0f) continue;
          pm = fmn(pm, alpha_margin(fmn(0.99f, co[3] * std::exp(power))));
        }
        flagged = pm < flag_eps;
      }
      float T_final = 1.0f - out_alpha[pix];
      float T = T_final;
      float g0 = grad_color[pix], g1 = grad_color[npix + pix], g2 = grad_color[2 * npix + pix];
      float gd = compute_depth ? grad_depth[pix] : 0.0f;
      float ga = grad_alpha[pix];
      float bg_dot = bg[0] * g0 + bg[1] * g1 + bg[2] * g2;
      float ar0 = 0, ar1 = 0, ar2 = 0, adr = 0, aar = 0, la = 0, lc0 = 0, lc1 = 0, lc2 = 0, ld = 0;
      float fx = (float)pxi, fy = (float)pyi;
      float m = 1.0f;
      for (int pos = lc - 1; pos >= 0; --pos) {
        int id = point_list[start + pos];
        const float* co = conic_opacity + id * 4;
        float d_x = xy[id * 2] - fx;
        float d_y = xy[id * 2 + 1] - fy;
        float power = -0.5f * (co[0] * d_x * d_x + co[2] * d_y * d_y) - co[1] * d_x * d_y;
        const float pmg = (margin || flagged) ? power_margin(power, co[0], co[1], co[2], d_x, d_y) : 1.0f;
        if (margin) m = fmn(m, pmg);
        // In a flagged pixel, a pair skipped by a decision within flag_eps of
        // its threshold may be taken by another exp implementation: its terms
        // are evaluated as if taken and counted in flagged_abs only (the
        // pixel's state is not advanced).
        if (power > 0.0f && !(flagged && pmg < flag_eps)) continue;
        // G = exp(power) and alpha = min(0.99, op * exp(power)) (backward_kernels.py:629-630):
        // one evaluation serves both, the same value
        float G = std::exp(power);
        float alpha = fmn(0.99f, co[3] * G);
        if (margin) m = fmn(m, alpha_margin(alpha));
        const bool take = power <= 0.0f && alpha >= (1.0f / 255.0f);
        if (!take && !(flagged && (pmg < flag_eps || alpha_margin(alpha) < flag_eps))) continue;
        // working copy of the back-to-front state, committed when the pair is taken
        float nT = T, nar0 = ar0, nar1 = ar1, nar2 = ar2, nadr = adr, naar = aar, nla = la, nld = ld;
        float nlc0 = lc0, nlc1 = lc1, nlc2 = lc2;
        float oma = fmx(1.0f - alpha, ONE_MINUS_ALPHA_MIN);
        nT = nT / oma;
        float dchannel = alpha * nT;
        float cr = features[id * 3], cg = features[id * 3 + 1], cb = features[id * 3 + 2];
        nar0 = nla * nlc0 + (1.0f - nla) * nar0;
        nar1 = nla * nlc1 + (1.0f - nla) * nar1;
        nar2 = nla * nlc2 + (1.0f - nla) * nar2;
        nlc0 = cr; nlc1 = cg; nlc2 = cb;
        float dL_dopa = (cr - nar0) * g0 + (cg - nar1) * g1 + (cb - nar2) * g2;
        float gf0 = dchannel * g0, gf1 = dchannel * g1, gf2 = dchannel * g2;
        float gdep = 0.0f;
        if (compute_depth) {
          float dv = depths[id];
          nadr = nla * nld + (1.0f - nla) * nadr;
          nld = dv;
          dL_dopa = dL_dopa + (dv - nadr) * gd;
          gdep = dchannel * gd;
        }
        naar = nla + (1.0f - nla) * naar;
        dL_dopa = dL_dopa + (1.0f - naar) * ga;
        dL_dopa = dL_dopa * nT;
        nla = alpha;
        dL_dopa = dL_dopa + (-T_final / oma) * bg_dot;
        float dL_dG = co[3] * dL_dopa;
        float gdx = G * d_x, gdy = G * d_y;
        float dG_ddelx = -gdx * co[0] - gdy * co[1];
        float dG_ddely = -gdy * co[2] - gdx * co[1];
        float v[10];
        v[0] = dL_dG * dG_ddelx * ddelx_dx;
        v[1] = dL_dG * dG_ddely * ddely_dy;
        v[2] = gdep;
        v[3] = -0.5f * gdx * d_x * dL_dG;
        v[4] = -0.5f * gdx * d_y * dL_dG;
        v[5] = -0.5f * gdy * d_y * dL_dG;
        v[6] = G * dL_dopa;
        v[7] = gf0; v[8] = gf1; v[9] = gf2;
        double* a = acc + (size_t)pos * ACC;
        if (!take) {
          for (int k = 0; k < 10; ++k) a[OFF_FLAG + k] += std::fabs((double)v[k]);
          continue;
        }
        T = nT; ar0 = nar0; ar1 = nar1; ar2 = nar2; adr = nadr; aar = naar; la = nla; ld = nld;
        lc0 = nlc0; lc1 = nlc1; lc2 = nlc2;
        for (int k = 0; k < 10; ++k) a[k] += (double)v[k];
        if (grad_abs)
          for (int k = 0; k < 10; ++k) a[OFF_ABS + k] += std::fabs((double)v[k]);
        if (cond_abs) {
          const double sc = power_scale(co[0], co[1], co[2], d_x, d_y);
          for (int k = 0; k < 10; ++k) a[OFF_COND + k] += std::fabs((double)v[k]) * sc;
        }
        if (flagged)
          for (int k = 0; k < 10; ++k) a[OFF_FLAG + k] += std::fabs((double)v[k]);
      }
      if (margin) margin[pix] = m;
    }
  }
  // Per-Gaussian totals, tile by tile in tile order (deterministic); each thread owns a range of
  // Gaussian ids and walks the whole list.
  static std::vector<double> g_sum, g_abs;
  if (g_sum.size() < (size_t)P * 10) g_sum.resize((size_t)P * 10);
  if (grad_abs && g_abs.size() < (size_t)P * 10) g_abs.resize((size_t)P * 10);
  // cond_abs is summed straight into the caller's array
  double* const sum = g_sum.data();
  double* const abs_sum = g_abs.data();
#pragma omp parallel
  {
    const int nth = omp_get_num_threads(), th = omp_get_thread_num();
    const long long lo_id = (long long)P * th / nth, hi_id = (long long)P * (th + 1) / nth;
    std::fill(sum + lo_id * 10, sum + hi_id * 10, 0.0);
    if (grad_abs) std::fill(abs_sum + lo_id * 10, abs_sum + hi_id * 10, 0.0);
    if (flagged_abs) std::fill(flagged_abs + lo_id * 10, flagged_abs + hi_id * 10, 0.0);
    if (cond_abs) std::fill(cond_abs + lo_id * 10, cond_abs + hi_id * 10, 0.0);
    for (int tile = 0; tile < ntile; ++tile) {
      const int start = ranges[2 * tile];
      const int n = ranges[2 * tile + 1] - start;
      if (n <= 0) continue;
      const double* const acc = acc_all + (size_t)start * ACC;
      for (int pos = 0; pos < n; ++pos) {
        const int id = point_list[start + pos];
        if (id < lo_id || id >= hi_id) continue;
        const double* a = &acc[(size_t)pos * ACC];
        for (int k = 0; k < 10; ++k) sum[(size_t)id * 10 + k] += a[k];
        if (grad_abs)
          for (int k = 0; k < 10; ++k) abs_sum[(size_t)id * 10 + k] += a[OFF_ABS + k];
        if (flagged_abs)
          for (int k = 0; k < 10; ++k) flagged_abs[(size_t)id * 10 + k] += a[OFF_FLAG + k];
        if (cond_abs)
          for (int k = 0; k < 10; ++k) cond_abs[(size_t)id * 10 + k] += a[OFF_COND + k];
      }
    }
  }
  for (int i = 0; i < P; ++i) {
    const double* s = &sum[(size_t)i * 10];
    grad_xy[i * 2] = (float)s[0];
    grad_xy[i * 2 + 1] = (float)s[1];
    grad_depths[i] = (float)s[2];
    for (int k = 0; k < 4; ++k) grad_co[i * 4 + k] = (float)s[3 + k];
    for (int k = 0; k < 3; ++k) grad_rgb[i * 3 + k] = (float)s[7 + k];
    if (grad_abs)
      for (int k = 0; k < 10; ++k) grad_abs[(size_t)i * 10 + k] = abs_sum[(size_t)i * 10 + k];
  }
}

// ---------------------------------------------------------------------------
// Preprocess + SH backward, scale/rotation path:
// backward_kernels.py:52-295 (fused) and :297-536 (SH).  Inputs are the render
// gradients (grad_xy etc.) and the user's gradients of the meta outputs.
// sh == nullptr -> colors_precomp path (no SH gradient, no SH mean term).
// cov3d_precomp != nullptr -> cov3D_precomp path: grad_cov3d is written and
// grad_scales/rotations are zero (backward_kernels.py:709-949,
// backward_ops.py:690-744).
// ---------------------------------------------------------------------------
namespace {
inline void dnormvdv(const float* v, const float* g, float* out) {
  // math_kernels.py:89-97
  float sum2 = v[0] * v[0] + v[1] * v[1] + v[2] * v[2];
  float invsum32 = 1.0f / std::sqrt(fmx(sum2 * sum2 * sum2, 1.0e-20f));
  out[0] = ((sum2 - v[0] * v[0]) * g[0] - v[1] * v[0] * g[1] - v[2] * v[0] * g[2]) * invsum32;
  out[1] = (-v[0] * v[1] * g[0] + (sum2 - v[1] * v[1]) * g[1] - v[2] * v[1] * g[2]) * invsum32;
  out[2] = (-v[0] * v[2] * g[0] - v[1] * v[2] * g[1] + (sum2 - v[2] * v[2]) * g[2]) * invsum32;
}

// backward_kernels.py:297-398 (v3 SoA kernel, degree >= 2) and :400-536
// (scalar kernel, degree <= 1); both evaluate the same expressions.
inline void sh_backward(const float* mean, const float* campos, const float* sp, int degree,
                        int K, const float* grad_rgb_in, const int* clamped, float* grad_sh,
                        float* grad_mean) {
  float dir[3] = {mean[0] - campos[0], mean[1] - campos[1], mean[2] - campos[2]};
  float len_sq = dir[0] * dir[0] + dir[1] * dir[1] + dir[2] * dir[2];
  float inv_len = 1.0f / std::sqrt(fmx(len_sq, 1.0e-20f));
  float x = dir[0] * inv_len, y = dir[1] * inv_len, z = dir[2] * inv_len;
  float g[3];
  for (int c = 0; c < 3; ++c) g[c] = grad_rgb_in[c] * (1.0f - (float)clamped[c]);
  float dx[3] = {0, 0, 0}, dy[3] = {0, 0, 0}, dz[3] = {0, 0, 0};
  for (int k = 0; k < K * 3; ++k) grad_sh[k] = 0.0f;
  if (K > 0)
    for (int c = 0; c < 3; ++c) grad_sh[c] = SH_C0 * g[c];
  if (degree > 0 && K > 3) {
    float b1 = -SH_C1 * y, b2 = SH_C1 * z, b3 = -SH_C1 * x;
    for (int c = 0; c < 3; ++c) {
      grad_sh[3 + c] = b1 * g[c];
      grad_sh[6 + c] = b2 * g[c];
      grad_sh[9 + c] = b3 * g[c];
      dx[c] = -SH_C1 * sp[9 + c];
      dy[c] = -SH_C1 * sp[3 + c];
      dz[c] = SH_C1 * sp[6 + c];
    }
    if (degree > 1 && K > 8) {
      float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      float w4 = SH_C2_0 * xy, w5 = SH_C2_1 * yz, w6 = SH_C2_2 * (2.0f * zz - xx - yy);
      float w7 = SH_C2_3 * xz, w8 = SH_C2_4 * (xx - yy);
      for (int c = 0; c < 3; ++c) {
        grad_sh[12 + c] = w4 * g[c];
        grad_sh[15 + c] = w5 * g[c];
        grad_sh[18 + c] = w6 * g[c];
        grad_sh[21 + c] = w7 * g[c];
        grad_sh[24 + c] = w8 * g[c];
        float s4 = sp[12 + c], s5 = sp[15 + c], s6 = sp[18 + c], s7 = sp[21 + c], s8 = sp[24 + c];
        dx[c] = dx[c] + (SH_C2_0 * y) * s4 + (SH_C2_2 * (-2.0f * x)) * s6 + (SH_C2_3 * z) * s7 +
                (SH_C2_4 * (2.0f * x)) * s8;
        dy[c] = dy[c] + (SH_C2_0 * x) * s4 + (SH_C2_1 * z) * s5 + (SH_C2_2 * (-2.0f * y)) * s6 +
                (SH_C2_4 * (-2.0f * y)) * s8;
        dz[c] = dz[c] + (SH_C2_1 * y) * s5 + (SH_C2_2 * (4.0f * z)) * s6 + (SH_C2_3 * x) * s7;
      }
      if (degree > 2 && K > 15) {
        float w9 = SH_C3_0 * y * (3.0f * xx - yy);
        float w10 = SH_C3_1 * xy * z;
        float w11 = SH_C3_2 * y * (4.0f * zz - xx - yy);
        float w12 = SH_C3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
        float w13 = SH_C3_4 * x * (4.0f * zz - xx - yy);
        float w14 = SH_C3_5 * z * (xx - yy);
        float w15 = SH_C3_6 * x * (xx - 3.0f * yy);
        for (int c = 0; c < 3; ++c) {
          grad_sh[27 + c] = w9 * g[c];
          grad_sh[30 + c] = w10 * g[c];
          grad_sh[33 + c] = w11 * g[c];
          grad_sh[36 + c] = w12 * g[c];
          grad_sh[39 + c] = w13 * g[c];
          grad_sh[42 + c] = w14 * g[c];
          grad_sh[45 + c] = w15 * g[c];
          float s9 = sp[27 + c], s10 = sp[30 + c], s11 = sp[33 + c], s12 = sp[36 + c],
                s13 = sp[39 + c], s14 = sp[42 + c], s15 = sp[45 + c];
          dx[c] = dx[c] + (SH_C3_0 * (6.0f * xy)) * s9 + (SH_C3_1 * yz) * s10 +
                  (SH_C3_2 * (-2.0f * xy)) * s11 + (SH_C3_3 * (-6.0f * xz)) * s12 +
                  (SH_C3_4 * (-3.0f * xx + 4.0f * zz - yy)) * s13 + (SH_C3_5 * (2.0f * xz)) * s14 +
                  (SH_C3_6 * (3.0f * (xx - yy))) * s15;
          dy[c] = dy[c] + (SH_C3_0 * (3.0f * (xx - yy))) * s9 + (SH_C3_1 * xz) * s10 +
                  (SH_C3_2 * (-3.0f * yy + 4.0f * zz - xx)) * s11 + (SH_C3_3 * (-6.0f * yz)) * s12 +
                  (SH_C3_4 * (-2.0f * xy)) * s13 + (SH_C3_5 * (-2.0f * yz)) * s14 +
                  (SH_C3_6 * (-6.0f * xy)) * s15;
          dz[c] = dz[c] + (SH_C3_1 * xy) * s10 + (SH_C3_2 * (8.0f * yz)) * s11 +
                  (SH_C3_3 * (3.0f * (2.0f * zz - xx - yy))) * s12 + (SH_C3_4 * (8.0f * xz)) * s13 +
                  (SH_C3_5 * (xx - yy)) * s14;
        }
      }
    }
  }
  float ddir[3];
  ddir[0] = dx[0] * g[0] + dx[1] * g[1] + dx[2] * g[2];
  ddir[1] = dy[0] * g[0] + dy[1] * g[1] + dy[2] * g[2];
  ddir[2] = dz[0] * g[0] + dz[1] * g[1] + dz[2] * g[2];
  dnormvdv(dir, ddir, grad_mean);
}
// cov3D_precomp backward: _backward_projected_means_warp_kernel
// (backward_kernels.py:842-875), _backward_cov2d_warp_kernel (:709-840) and
// _fused_backward_accumulate_warp_kernel (:34-50), as composed by
// backward_ops.py:690-744.  Gaussians with radius <= 0 keep the zero
// cov-gradient and zero cov mean-gradient of the torch.zeros buffers.
inline void precomp_backward(int tid, const float* mean, int rad, const float* c3, const float* vf,
                             const float* pr, float tanfovx, float tanfovy, float focal_x,
                             float focal_y, const float* render_grad_xy,
                             const float* render_grad_depth, const float* render_grad_co,
                             const float* render_grad_rgb, const float* grad_proj_2d,
                             const float* grad_conic_2d, const float* grad_conic_2d_inv,
                             const float* sh, int degree, int K, const float* campos,
                             const int* clamped, float* grad_means3d, float* grad_means2d,
                             float* grad_opacity, float* grad_sh, float* grad_colors,
                             float* grad_cov3d) {
  // projected means
  float hom_x = pr[0] * mean[0] + pr[4] * mean[1] + pr[8] * mean[2] + pr[12];
  float hom_y = pr[1] * mean[0] + pr[5] * mean[1] + pr[9] * mean[2] + pr[13];
  float hom_w = pr[3] * mean[0] + pr[7] * mean[1] + pr[11] * mean[2] + pr[15];
  float inv_w = 1.0f / (hom_w + 1.0e-7f);
  float mul1 = hom_x * inv_w * inv_w;
  float mul2 = hom_y * inv_w * inv_w;
  float g0 = render_grad_xy[tid * 2], g1 = render_grad_xy[tid * 2 + 1];
  if (rad > 0) {
    g0 = g0 + grad_proj_2d[tid * 2];
    g1 = g1 + grad_proj_2d[tid * 2 + 1];
  }
  float ox = (pr[0] * inv_w - pr[3] * mul1) * g0 + (pr[1] * inv_w - pr[3] * mul2) * g1;
  float oy = (pr[4] * inv_w - pr[7] * mul1) * g0 + (pr[5] * inv_w - pr[7] * mul2) * g1;
  float oz = (pr[8] * inv_w - pr[11] * mul1) * g0 + (pr[9] * inv_w - pr[11] * mul2) * g1;
  float mul3 = vf[2] * mean[0] + vf[6] * mean[1] + vf[10] * mean[2] + vf[14];
  float dg = render_grad_depth[tid];
  ox = ox + (vf[2] - vf[3] * mul3) * dg;
  oy = oy + (vf[6] - vf[7] * mul3) * dg;
  oz = oz + (vf[10] - vf[11] * mul3) * dg;
  // cov2d backward
  float gm[3] = {0, 0, 0};
  float gc[6] = {0, 0, 0, 0, 0, 0};
  if (rad > 0) {
    float x = vf[0] * mean[0] + vf[4] * mean[1] + vf[8] * mean[2] + vf[12];
    float y = vf[1] * mean[0] + vf[5] * mean[1] + vf[9] * mean[2] + vf[13];
    float z = vf[2] * mean[0] + vf[6] * mean[1] + vf[10] * mean[2] + vf[14];
    float limx = 1.3f * tanfovx, limy = 1.3f * tanfovy;
    float txtz = x / z, tytz = y / z;
    float tx = fclamp(txtz, -limx, limx) * z;
    float ty = fclamp(tytz, -limy, limy) * z;
    float xm = 1.0f, ym = 1.0f;
    if (txtz < -limx || txtz > limx) xm = 0.0f;
    if (tytz < -limy || tytz > limy) ym = 0.0f;
    float j00 = focal_x / z;
    float j02 = -(focal_x * tx) / (z * z);
    float j11 = focal_y / z;
    float j12 = -(focal_y * ty) / (z * z);
    float w00 = vf[0], w01 = vf[1], w02 = vf[2], w10 = vf[4], w11 = vf[5], w12 = vf[6];
    float w20 = vf[8], w21 = vf[9], w22 = vf[10];
    float t00 = w00 * j00 + w02 * j02, t10 = w10 * j00 + w12 * j02, t20 = w20 * j00 + w22 * j02;
    float t01 = w01 * j11 + w02 * j12, t11 = w11 * j11 + w12 * j12, t21 = w21 * j11 + w22 * j12;
    float v00 = c3[0], v01 = c3[1], v02 = c3[2], v11 = c3[3], v12 = c3[4], v22 = c3[5];
    float vt0x = v00 * t00 + v01 * t10 + v02 * t20;
    float vt0y = v01 * t00 + v11 * t10 + v12 * t20;
    float vt0z = v02 * t00 + v12 * t10 + v22 * t20;
    float vt1x = v00 * t01 + v01 * t11 + v02 * t21;
    float vt1y = v01 * t01 + v11 * t11 + v12 * t21;
    float vt1z = v02 * t01 + v12 * t11 + v22 * t21;
    const float filt = 0.0f;
    float a = t00 * vt0x + t10 * vt0y + t20 * vt0z + 0.3f + filt;
    float b = t00 * vt1x + t10 * vt1y + t20 * vt1z;
    float c = t01 * vt1x + t11 * vt1y + t21 * vt1z + 0.3f + filt;
    float denom = a * c - b * b;
    float d2i = 1.0f / (denom * denom + 1.0e-7f);
    float tc0 = render_grad_co[tid * 4 + 0] + grad_conic_2d[tid * 3 + 0];
    float tc1 = render_grad_co[tid * 4 + 1] + grad_conic_2d[tid * 3 + 1];
    float tc2 = render_grad_co[tid * 4 + 2] + grad_conic_2d[tid * 3 + 2];
    float dL_da = d2i * (-c * c * tc0 + 2.0f * b * c * tc1 + (denom - a * c) * tc2);
    float dL_dc = d2i * (-a * a * tc2 + 2.0f * a * b * tc1 + (denom - a * c) * tc0);
    float dL_db = d2i * 2.0f * (b * c * tc0 - (denom + 2.0f * b * b) * tc1 + a * b * tc2);
    dL_da = dL_da + grad_conic_2d_inv[tid * 3 + 0];
    dL_db = dL_db + grad_conic_2d_inv[tid * 3 + 1];
    dL_dc = dL_dc + grad_conic_2d_inv[tid * 3 + 2];
    gc[0] = t00 * t00 * dL_da + t00 * t01 * dL_db + t01 * t01 * dL_dc;
    gc[3] = t10 * t10 * dL_da + t10 * t11 * dL_db + t11 * t11 * dL_dc;
    gc[5] = t20 * t20 * dL_da + t20 * t21 * dL_db + t21 * t21 * dL_dc;
    gc[1] = 2.0f * t00 * t10 * dL_da + (t00 * t11 + t01 * t10) * dL_db + 2.0f * t01 * t11 * dL_dc;
    gc[2] = 2.0f * t00 * t20 * dL_da + (t00 * t21 + t01 * t20) * dL_db + 2.0f * t01 * t21 * dL_dc;
    gc[4] = 2.0f * t10 * t20 * dL_da + (t10 * t21 + t11 * t20) * dL_db + 2.0f * t11 * t21 * dL_dc;
    float dT00 = 2.0f * (t00 * v00 + t10 * v01 + t20 * v02) * dL_da + (t01 * v00 + t11 * v01 + t21 * v02) * dL_db;
    float dT01 = 2.0f * (t00 * v01 + t10 * v11 + t20 * v12) * dL_da + (t01 * v01 + t11 * v11 + t21 * v12) * dL_db;
    float dT02 = 2.0f * (t00 * v02 + t10 * v12 + t20 * v22) * dL_da + (t01 * v02 + t11 * v12 + t21 * v22) * dL_db;
    float dT10 = 2.0f * (t01 * v00 + t11 * v01 + t21 * v02) * dL_dc + (t00 * v00 + t10 * v01 + t20 * v02) * dL_db;
    float dT11 = 2.0f * (t01 * v01 + t11 * v11 + t21 * v12) * dL_dc + (t00 * v01 + t10 * v11 + t20 * v12) * dL_db;
    float dT12 = 2.0f * (t01 * v02 + t11 * v12 + t21 * v22) * dL_dc + (t00 * v02 + t10 * v12 + t20 * v22) * dL_db;
    float dJ00 = w00 * dT00 + w10 * dT01 + w20 * dT02;
    float dJ02 = w02 * dT00 + w12 * dT01 + w22 * dT02;
    float dJ11 = w01 * dT10 + w11 * dT11 + w21 * dT12;
    float dJ12 = w02 * dT10 + w12 * dT11 + w22 * dT12;
    float tz_inv = 1.0f / z;
    float tz2 = tz_inv * tz_inv;
    float tz3 = tz2 * tz_inv;
    float dL_dtx = xm * -focal_x * tz2 * dJ02;
    float dL_dty = ym * -focal_y * tz2 * dJ12;
    float dL_dtz = -focal_x * tz2 * dJ00 - focal_y * tz2 * dJ11 + (2.0f * focal_x * tx) * tz3 * dJ02 +
                   (2.0f * focal_y * ty) * tz3 * dJ12;
    gm[0] = vf[0] * dL_dtx + vf[1] * dL_dty + vf[2] * dL_dtz;
    gm[1] = vf[4] * dL_dtx + vf[5] * dL_dty + vf[6] * dL_dtz;
    gm[2] = vf[8] * dL_dtx + vf[9] * dL_dty + vf[10] * dL_dtz;
  }
  float gsm[3] = {0, 0, 0};
  if (sh)
    sh_backward(mean, campos, sh + (size_t)tid * K * 3, degree, K, render_grad_rgb + tid * 3,
                clamped + tid * 3, grad_sh + (size_t)tid * K * 3, gsm);
  float a0 = ox + gm[0], a1 = oy + gm[1], a2 = oz + gm[2];
  if (sh) {
    a0 = a0 + gsm[0];
    a1 = a1 + gsm[1];
    a2 = a2 + gsm[2];
  }
  grad_means3d[tid * 3] = a0;
  grad_means3d[tid * 3 + 1] = a1;
  grad_means3d[tid * 3 + 2] = a2;
  grad_means2d[tid * 3] = render_grad_xy[tid * 2];
  grad_means2d[tid * 3 + 1] = render_grad_xy[tid * 2 + 1];
  grad_means2d[tid * 3 + 2] = 0.0f;
  if (grad_cov3d)
    for (int k = 0; k < 6; ++k) grad_cov3d[tid * 6 + k] = gc[k];
  grad_opacity[tid] = render_grad_co[tid * 4 + 3];
  if (grad_colors)
    for (int k = 0; k < 3; ++k) grad_colors[tid * 3 + k] = render_grad_rgb[tid * 3 + k];
}
}  // namespace

OR_EXPORT void or_preprocess_bwd(
    int P, const float* means, const int* radii, const float* scales, const float* rotations,
    float scale_modifier, const float* cov3d_precomp, const float* view, const float* proj,
    float tanfovx, float tanfovy, float focal_x, float focal_y,
    const float* render_grad_xy, const float* render_grad_depth, const float* render_grad_co,
    const float* render_grad_rgb, const float* grad_proj_2d, const float* grad_conic_2d,
    const float* grad_conic_2d_inv, const float* sh, int degree, int K, const float* campos,
    const int* clamped,
    // outputs
    float* grad_means3d, float* grad_means2d, float* grad_scales, float* grad_rotations,
    float* grad_opacity, float* grad_sh, float* grad_colors, float* grad_cov3d) {
  const float* pr = proj;
  const float* vf = view;
#pragma omp parallel for schedule(static)
  for (int tid = 0; tid < P; ++tid) {
    const float* mean = means + tid * 3;
    int rad = radii[tid];
    if (cov3d_precomp) {
      precomp_backward(tid, mean, rad, cov3d_precomp + tid * 6, vf, pr, tanfovx, tanfovy, focal_x,
                       focal_y, render_grad_xy, render_grad_depth, render_grad_co, render_grad_rgb,
                       grad_proj_2d, grad_conic_2d, grad_conic_2d_inv, sh, degree, K, campos,
                       clamped, grad_means3d, grad_means2d, grad_opacity, grad_sh, grad_colors,
                       grad_cov3d);
      if (grad_scales)
        for (int k = 0; k < 3; ++k) grad_scales[tid * 3 + k] = 0.0f;
      if (grad_rotations)
        for (int k = 0; k < 4; ++k) grad_rotations[tid * 4 + k] = 0.0f;
      continue;
    }
    // ---- Part A: projected means (backward_kernels.py:89-112) ----
    float hom_x = pr[0] * mean[0] + pr[4] * mean[1] + pr[8] * mean[2] + pr[12];
    float hom_y = pr[1] * mean[0] + pr[5] * mean[1] + pr[9] * mean[2] + pr[13];
    float hom_w = pr[3] * mean[0] + pr[7] * mean[1] + pr[11] * mean[2] + pr[15];
    float inv_w = 1.0f / (hom_w + 1.0e-7f);
    float gxy0 = render_grad_xy[tid * 2], gxy1 = render_grad_xy[tid * 2 + 1];
    float inv_w2 = inv_w * inv_w;
    if (rad > 0) {
      gxy0 = gxy0 + grad_proj_2d[tid * 2];
      gxy1 = gxy1 + grad_proj_2d[tid * 2 + 1];
    }
    float gh = hom_x * gxy0 + hom_y * gxy1;
    float pm_x = inv_w * (pr[0] * gxy0 + pr[1] * gxy1) - pr[3] * inv_w2 * gh;
    float pm_y = inv_w * (pr[4] * gxy0 + pr[5] * gxy1) - pr[7] * inv_w2 * gh;
    float pm_z = inv_w * (pr[8] * gxy0 + pr[9] * gxy1) - pr[11] * inv_w2 * gh;
    float zz = vf[2] * mean[0] + vf[6] * mean[1] + vf[10] * mean[2] + vf[14];
    float dgrad = render_grad_depth[tid];
    pm_x = pm_x + (vf[2] - vf[3] * zz) * dgrad;
    pm_y = pm_y + (vf[6] - vf[7] * zz) * dgrad;
    pm_z = pm_z + (vf[10] - vf[11] * zz) * dgrad;

    // ---- Part B: cov2d -> cov3d -> scale/rotation (backward_kernels.py:114-287) ----
    float gcm0 = 0, gcm1 = 0, gcm2 = 0;
    float gs[3] = {0, 0, 0}, gr[4] = {0, 0, 0, 0}, gc3[6] = {0, 0, 0, 0, 0, 0};
    if (rad > 0) {
      float x = vf[0] * mean[0] + vf[4] * mean[1] + vf[8] * mean[2] + vf[12];
      float y = vf[1] * mean[0] + vf[5] * mean[1] + vf[9] * mean[2] + vf[13];
      float z = vf[2] * mean[0] + vf[6] * mean[1] + vf[10] * mean[2] + vf[14];
      float tz_inv = 1.0f / (z + 1.0e-7f);
      float limx = 1.3f * tanfovx, limy = 1.3f * tanfovy;
      float txtz = x * tz_inv, tytz = y * tz_inv;
      float x_mul = 1.0f, y_mul = 1.0f;
      if (txtz < -limx || txtz > limx) x_mul = 0.0f;
      if (tytz < -limy || tytz > limy) y_mul = 0.0f;
      float tx = fclamp(txtz, -limx, limx), ty = fclamp(tytz, -limy, limy);
      float j00 = focal_x * tz_inv;
      float j02 = -j00 * tx;
      float j11 = focal_y * tz_inv;
      float j12 = -j11 * ty;
      float w00 = vf[0], w01 = vf[1], w02 = vf[2], w10 = vf[4], w11 = vf[5], w12 = vf[6];
      float w20 = vf[8], w21 = vf[9], w22 = vf[10];
      float t00 = w00 * j00 + w02 * j02, t10 = w10 * j00 + w12 * j02, t20 = w20 * j00 + w22 * j02;
      float t01 = w01 * j11 + w02 * j12, t11 = w11 * j11 + w12 * j12, t21 = w21 * j11 + w22 * j12;
      float V[6];
      MRows mm{};
      if (cov3d_precomp) {
        for (int k = 0; k < 6; ++k) V[k] = cov3d_precomp[tid * 6 + k];
      } else {
        // The reference reads the cov3d the forward wrote; recomputing it
        // with the same expressions gives the same bits.
        mm = make_m(scales + tid * 3, rotations + tid * 4, scale_modifier);
        V[0] = mm.m00 * mm.m00 + mm.m10 * mm.m10 + mm.m20 * mm.m20;
        V[1] = mm.m00 * mm.m01 + mm.m10 * mm.m11 + mm.m20 * mm.m21;
        V[2] = mm.m00 * mm.m02 + mm.m10 * mm.m12 + mm.m20 * mm.m22;
        V[3] = mm.m01 * mm.m01 + mm.m11 * mm.m11 + mm.m21 * mm.m21;
        V[4] = mm.m01 * mm.m02 + mm.m11 * mm.m12 + mm.m21 * mm.m22;
        V[5] = mm.m02 * mm.m02 + mm.m12 * mm.m12 + mm.m22 * mm.m22;
      }
      float v00 = V[0], v01 = V[1], v02 = V[2], v11 = V[3], v12 = V[4], v22 = V[5];
      float vt0x = v00 * t00 + v01 * t10 + v02 * t20;
      float vt0y = v01 * t00 + v11 * t10 + v12 * t20;
      float vt0z = v02 * t00 + v12 * t10 + v22 * t20;
      float vt1x = v00 * t01 + v01 * t11 + v02 * t21;
      float vt1y = v01 * t01 + v11 * t11 + v12 * t21;
      float vt1z = v02 * t01 + v12 * t11 + v22 * t21;
      const float filt = 0.0f;  // cov2d_filter_variance (backward_ops.py:479)
      float aa = t00 * vt0x + t10 * vt0y + t20 * vt0z + 0.3f + filt;
      float bb = t00 * vt1x + t10 * vt1y + t20 * vt1z;
      float cc = t01 * vt1x + t11 * vt1y + t21 * vt1z + 0.3f + filt;
      float denom = aa * cc - bb * bb;
      float denom2inv = 1.0f / (denom * denom + 1.0e-7f);
      float tc0 = render_grad_co[tid * 4 + 0] + grad_conic_2d[tid * 3 + 0];
      float tc1 = render_grad_co[tid * 4 + 1] + grad_conic_2d[tid * 3 + 1];
      float tc2 = render_grad_co[tid * 4 + 2] + grad_conic_2d[tid * 3 + 2];
      float dL_da = denom2inv * (-cc * cc * tc0 + 2.0f * bb * cc * tc1 - bb * bb * tc2);
      float dL_dc = denom2inv * (-aa * aa * tc2 + 2.0f * aa * bb * tc1 - bb * bb * tc0);
      float dL_db = denom2inv * 2.0f * (bb * cc * tc0 - (aa * cc + bb * bb) * tc1 + aa * bb * tc2);
      dL_da = dL_da + grad_conic_2d_inv[tid * 3 + 0];
      dL_db = dL_db + grad_conic_2d_inv[tid * 3 + 1];
      dL_dc = dL_dc + grad_conic_2d_inv[tid * 3 + 2];
      float gc0 = t00 * t00 * dL_da + t00 * t01 * dL_db + t01 * t01 * dL_dc;
      float gc3v = t10 * t10 * dL_da + t10 * t11 * dL_db + t11 * t11 * dL_dc;
      float gc5 = t20 * t20 * dL_da + t20 * t21 * dL_db + t21 * t21 * dL_dc;
      float gc1 = 2.0f * t00 * t10 * dL_da + (t00 * t11 + t01 * t10) * dL_db + 2.0f * t01 * t11 * dL_dc;
      float gc2 = 2.0f * t00 * t20 * dL_da + (t00 * t21 + t01 * t20) * dL_db + 2.0f * t01 * t21 * dL_dc;
      float gc4 = 2.0f * t10 * t20 * dL_da + (t10 * t21 + t11 * t20) * dL_db + 2.0f * t11 * t21 * dL_dc;
      float dT00 = 2.0f * vt0x * dL_da + vt1x * dL_db;
      float dT01 = 2.0f * vt0y * dL_da + vt1y * dL_db;
      float dT02 = 2.0f * vt0z * dL_da + vt1z * dL_db;
      float dT10 = vt0x * dL_db + 2.0f * vt1x * dL_dc;
      float dT11 = vt0y * dL_db + 2.0f * vt1y * dL_dc;
      float dT12 = vt0z * dL_db + 2.0f * vt1z * dL_dc;
      float dJ00 = w00 * dT00 + w10 * dT01 + w20 * dT02;
      float dJ02 = w02 * dT00 + w12 * dT01 + w22 * dT02;
      float dJ11 = w01 * dT10 + w11 * dT11 + w21 * dT12;
      float dJ12 = w02 * dT10 + w12 * dT11 + w22 * dT12;
      float dL_dtx = x_mul * -j00 * tz_inv * dJ02;
      float dL_dty = y_mul * -j11 * tz_inv * dJ12;
      float dL_dtz = -(j00 * dJ00 + j11 * dJ11 + 2.0f * j02 * dJ02 + 2.0f * j12 * dJ12) * tz_inv;
      gcm0 = w00 * dL_dtx + w01 * dL_dty + w02 * dL_dtz;
      gcm1 = w10 * dL_dtx + w11 * dL_dty + w12 * dL_dtz;
      gcm2 = w20 * dL_dtx + w21 * dL_dty + w22 * dL_dtz;
      if (cov3d_precomp) {
        gc3[0] = gc0; gc3[1] = gc1; gc3[2] = gc2; gc3[3] = gc3v; gc3[4] = gc4; gc3[5] = gc5;
      } else {
        float s0 = scales[tid * 3] * scale_modifier, s1 = scales[tid * 3 + 1] * scale_modifier,
              s2 = scales[tid * 3 + 2] * scale_modifier;
        const float* qq = rotations + tid * 4;
        float rr = qq[0], xq = qq[1], yq = qq[2], zq = qq[3];
        float sg00 = gc0, sg01 = 0.5f * gc1, sg02 = 0.5f * gc2, sg11 = gc3v, sg12 = 0.5f * gc4, sg22 = gc5;
        float dM00 = 2.0f * (mm.m00 * sg00 + mm.m01 * sg01 + mm.m02 * sg02);
        float dM01 = 2.0f * (mm.m00 * sg01 + mm.m01 * sg11 + mm.m02 * sg12);
        float dM02 = 2.0f * (mm.m00 * sg02 + mm.m01 * sg12 + mm.m02 * sg22);
        float dM10 = 2.0f * (mm.m10 * sg00 + mm.m11 * sg01 + mm.m12 * sg02);
        float dM11 = 2.0f * (mm.m10 * sg01 + mm.m11 * sg11 + mm.m12 * sg12);
        float dM12 = 2.0f * (mm.m10 * sg02 + mm.m11 * sg12 + mm.m12 * sg22);
        float dM20 = 2.0f * (mm.m20 * sg00 + mm.m21 * sg01 + mm.m22 * sg02);
        float dM21 = 2.0f * (mm.m20 * sg01 + mm.m21 * sg11 + mm.m22 * sg12);
        float dM22 = 2.0f * (mm.m20 * sg02 + mm.m21 * sg12 + mm.m22 * sg22);
        gs[0] = scale_modifier * (dM00 * mm.r00 + dM01 * mm.r01 + dM02 * mm.r02);
        gs[1] = scale_modifier * (dM10 * mm.r10 + dM11 * mm.r11 + dM12 * mm.r12);
        gs[2] = scale_modifier * (dM20 * mm.r20 + dM21 * mm.r21 + dM22 * mm.r22);
        float dR00 = dM00 * s0, dR01 = dM01 * s0, dR02 = dM02 * s0;
        float dR10 = dM10 * s1, dR11 = dM11 * s1, dR12 = dM12 * s1;
        float dR20 = dM20 * s2, dR21 = dM21 * s2, dR22 = dM22 * s2;
        gr[0] = 2.0f * zq * (dR01 - dR10) + 2.0f * yq * (dR20 - dR02) + 2.0f * xq * (dR12 - dR21);
        gr[1] = 2.0f * yq * (dR10 + dR01) + 2.0f * zq * (dR20 + dR02) + 2.0f * rr * (dR12 - dR21) -
                4.0f * xq * (dR22 + dR11);
        gr[2] = 2.0f * xq * (dR10 + dR01) + 2.0f * rr * (dR20 - dR02) + 2.0f * zq * (dR12 + dR21) -
                4.0f * yq * (dR22 + dR00);
        gr[3] = 2.0f * rr * (dR01 - dR10) + 2.0f * xq * (dR20 + dR02) + 2.0f * yq * (dR12 + dR21) -
                4.0f * zq * (dR11 + dR00);
      }
    }
    // ---- SH backward ----
    float gsm[3] = {0, 0, 0};
    if (sh) {
      sh_backward(mean, campos, sh + (size_t)tid * K * 3, degree, K, render_grad_rgb + tid * 3,
                  clamped + tid * 3, grad_sh + (size_t)tid * K * 3, gsm);
    }
    // ---- Part C: accumulate (backward_kernels.py:289-295) ----
    float a0 = pm_x + gcm0, a1 = pm_y + gcm1, a2 = pm_z + gcm2;
    if (sh) {
      a0 = a0 + gsm[0];
      a1 = a1 + gsm[1];
      a2 = a2 + gsm[2];
    }
    grad_means3d[tid * 3] = a0;
    grad_means3d[tid * 3 + 1] = a1;
    grad_means3d[tid * 3 + 2] = a2;
    grad_means2d[tid * 3] = render_grad_xy[tid * 2];
    grad_means2d[tid * 3 + 1] = render_grad_xy[tid * 2 + 1];
    grad_means2d[tid * 3 + 2] = 0.0f;
    if (grad_scales)
      for (int k = 0; k < 3; ++k) grad_scales[tid * 3 + k] = gs[k];
    if (grad_rotations)
      for (int k = 0; k < 4; ++k) grad_rotations[tid * 4 + k] = gr[k];
    if (grad_cov3d)
      for (int k = 0; k < 6; ++k) grad_cov3d[tid * 6 + k] = gc3[k];
    grad_opacity[tid] = render_grad_co[tid * 4 + 3];
    if (grad_colors)
      for (int k = 0; k < 3; ++k) grad_colors[tid * 3 + k] = render_grad_rgb[tid * 3 + k];
  }
}

// ---------------------------------------------------------------------------
// Fused SSIM (gswarp/fused_ssim.py).  11-tap Gaussian (sigma 1.5) weights as
// float32 constants (fused_ssim.py:47-57).  Forward train path 'same':
// _fwd_h (:461-518) + _fwd_v_train_tiled (:522-638); 'valid': _fwd_h +
// _fwd_v_train_valid (:760-828).  Backward 'same': _bwd_h_scalar (:831-874) +
// _bwd_v_tiled (:985-1067); 'valid': _bwd_h_scalar_valid (:878-935) + _bwd_v
// (:938-981).  ssim_sum receives the double-precision sum of the SSIM map
// over the padding's region (the reference takes torch.mean of it).
// ---------------------------------------------------------------------------
namespace {
const float GW[11] = {0.001028380123898387f, 0.0075987582094967365f, 0.036000773310661316f,
                      0.10936068743467331f,  0.21300552785396576f,   0.26601171493530273f,
                      0.21300552785396576f,  0.10936068743467331f,   0.036000773310661316f,
                      0.0075987582094967365f, 0.001028380123898387f};
}

OR_EXPORT void or_ssim_fwd(int B, int CH, int H, int W, const float* img1, const float* img2,
                           float C1, float C2, int valid, double* ssim_sum, float* ssim_map,
                           float* dm0, float* dm1, float* dm2) {
  const long long plane = (long long)H * W;
  const int planes = B * CH;
  std::vector<float> h((size_t)4 * plane * planes);
  float* h0 = h.data();
  float* h1 = h0 + plane * planes;
  float* h2 = h1 + plane * planes;
  float* h3 = h2 + plane * planes;
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < (long long)planes * H; ++row) {
    const long long base = row * W;
    for (int x = 0; x < W; ++x) {
      float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      for (int k = 0; k < 5; ++k) {
        int nl = x + k - 5, nr = x + 5 - k;
        float g = GW[k];
        float v1l = 0, v2l = 0, v1r = 0, v2r = 0;
        if (nl >= 0 && nl < W) { v1l = img1[base + nl]; v2l = img2[base + nl]; }
        if (nr >= 0 && nr < W) { v1r = img1[base + nr]; v2r = img2[base + nr]; }
        a0 = a0 + g * (v1l + v1r);
        a1 = a1 + g * (v2l + v2r);
        a2 = a2 + g * (v1l * v1l + v2l * v2l + v1r * v1r + v2r * v2r);
        a3 = a3 + g * (v1l * v2l + v1r * v2r);
      }
      float v1c = img1[base + x], v2c = img2[base + x];
      a0 = a0 + GW[5] * v1c;
      a1 = a1 + GW[5] * v2c;
      a2 = a2 + GW[5] * (v1c * v1c + v2c * v2c);
      a3 = a3 + GW[5] * v1c * v2c;
      h0[base + x] = a0; h1[base + x] = a1; h2[base + x] = a2; h3[base + x] = a3;
    }
  }
  double total = 0.0;
  const int y_lo = valid ? 5 : 0, y_hi = valid ? H - 5 : H;
  const int x_lo = valid ? 5 : 0, x_hi = valid ? W - 5 : W;
  const int Wv = valid ? W - 10 : W;
#pragma omp parallel for schedule(static) reduction(+ : total)
  for (long long prow = 0; prow < (long long)planes * H; ++prow) {
    int pl = (int)(prow / H), y = (int)(prow % H);
    if (y < y_lo || y >= y_hi) continue;
    const long long pbase = (long long)pl * plane;
    for (int x = x_lo; x < x_hi; ++x) {
      float a[4] = {0, 0, 0, 0};
      const float* hs[4] = {h0 + pbase, h1 + pbase, h2 + pbase, h3 + pbase};
      for (int k = 0; k < 5; ++k) {
        int top = y + k - 5, bot = y + 5 - k;
        float g = GW[k];
        if (valid) {
          for (int i = 0; i < 4; ++i)
            a[i] = a[i] + g * (hs[i][(long long)top * W + x] + hs[i][(long long)bot * W + x]);
        } else {
          if (top >= 0 && top < H)
            for (int i = 0; i < 4; ++i) a[i] = a[i] + g * hs[i][(long long)top * W + x];
          if (bot >= 0 && bot < H)
            for (int i = 0; i < 4; ++i) a[i] = a[i] + g * hs[i][(long long)bot * W + x];
        }
      }
      for (int i = 0; i < 4; ++i) a[i] = a[i] + GW[5] * hs[i][(long long)y * W + x];
      float mu1 = a[0], mu2 = a[1];
      float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu1mu2 = mu1 * mu2;
      float Av = mu1_sq + mu2_sq + C1;
      float Bv = a[2] - mu1_sq - mu2_sq + C2;
      float Cv = 2.0f * mu1mu2 + C1;
      float Dv = 2.0f * (a[3] - mu1mu2) + C2;
      float rA = 1.0f / Av, rB = 1.0f / Bv, rAB = rA * rB;
      float m = Cv * Dv * rAB;
      long long full = pbase + (long long)y * W + x;
      if (ssim_map) {
        long long oi = valid ? ((long long)pl * (H - 10) + (y - 5)) * Wv + (x - 5) : full;
        ssim_map[oi] = m;
      }
      if (dm0) {
        dm0[full] = 2.0f * (mu2 * (Dv - Cv) * rAB + mu1 * m * (rB - rA));
        dm1[full] = -m * rB;
        dm2[full] = 2.0f * Cv * rAB;
      }
      total += (double)m;
    }
  }
  *ssim_sum = total;
}

// grad = dL/dimg1 given dm maps from or_ssim_fwd; scale = inv_N * upstream
// computed in float32 exactly as the reference does.
OR_EXPORT void or_ssim_bwd(int B, int CH, int H, int W, const float* img1, const float* img2,
                           const float* dm0, const float* dm1, const float* dm2, float inv_n,
                           float upstream, int valid, float* grad) {
  const long long plane = (long long)H * W;
  const int planes = B * CH;
  std::vector<float> t((size_t)3 * plane * planes);
  float* t0 = t.data();
  float* t1 = t0 + plane * planes;
  float* t2 = t1 + plane * planes;
  const float scale = inv_n * upstream;
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < (long long)planes * H; ++row) {
    const long long base = row * W;
    int y = (int)(row % H);
    for (int x = 0; x < W; ++x) {
      float s0 = 0, s1 = 0, s2 = 0;
      if (valid && (y < 5 || y >= H - 5)) {
        t0[base + x] = 0; t1[base + x] = 0; t2[base + x] = 0;
        continue;
      }
      const int lo = valid ? 5 : 0, hi = valid ? W - 5 : W;
      for (int k = 0; k < 5; ++k) {
        int nl = x + k - 5, nr = x + 5 - k;
        float gs = GW[k] * scale;
        if (nl >= lo && nl < hi) {
          s0 = s0 + gs * dm0[base + nl]; s1 = s1 + gs * dm1[base + nl]; s2 = s2 + gs * dm2[base + nl];
        }
        if (nr >= lo && nr < hi) {
          s0 = s0 + gs * dm0[base + nr]; s1 = s1 + gs * dm1[base + nr]; s2 = s2 + gs * dm2[base + nr];
        }
      }
      if (!valid || (x >= 5 && x < W - 5)) {
        float gs = GW[5] * scale;
        s0 = s0 + gs * dm0[base + x]; s1 = s1 + gs * dm1[base + x]; s2 = s2 + gs * dm2[base + x];
      }
      t0[base + x] = s0; t1[base + x] = s1; t2[base + x] = s2;
    }
  }
#pragma omp parallel for schedule(static)
  for (long long prow = 0; prow < (long long)planes * H; ++prow) {
    int pl = (int)(prow / H), y = (int)(prow % H);
    const long long pbase = (long long)pl * plane;
    for (int x = 0; x < W; ++x) {
      float a0 = 0, a1 = 0, a2 = 0;
      for (int k = 0; k < 5; ++k) {
        int top = y + k - 5, bot = y + 5 - k;
        float g = GW[k];
        if (top >= 0 && top < H) {
          long long i = pbase + (long long)top * W + x;
          a0 = a0 + g * t0[i]; a1 = a1 + g * t1[i]; a2 = a2 + g * t2[i];
        }
        if (bot >= 0 && bot < H) {
          long long i = pbase + (long long)bot * W + x;
          a0 = a0 + g * t0[i]; a1 = a1 + g * t1[i]; a2 = a2 + g * t2[i];
        }
      }
      long long c = pbase + (long long)y * W + x;
      a0 = a0 + GW[5] * t0[c]; a1 = a1 + GW[5] * t1[c]; a2 = a2 + GW[5] * t2[c];
      grad[c] = a0 + 2.0f * img1[c] * a1 + img2[c] * a2;
    }
  }
}

// ---------------------------------------------------------------------------
// KNN initialiser (gswarp/knn.py:48-401): Morton codes, stable sort,
// 1024-point boxes, box-pruned 3-NN.  out[i] = mean of the three smallest
// squared distances to other points.  Requires P >= 4.
// ---------------------------------------------------------------------------
namespace {
inline uint32_t prep_morton(uint32_t x) {
  x = (x | (x << 16)) & 0x030000FFu;
  x = (x | (x << 8)) & 0x0300F00Fu;
  x = (x | (x << 4)) & 0x030C30C3u;
  x = (x | (x << 2)) & 0x09249249u;
  return x;
}
inline uint32_t f2u(float x) {  // cvt.rzi.u32.f32: saturating, NaN -> 0
  if (!(x > 0.0f)) return 0u;
  if (x >= 4294967296.0f) return 0xFFFFFFFFu;
  return (uint32_t)x;
}
inline float box_dist(const float* bmin, const float* bmax, float px, float py, float pz) {
  float dx = 0, dy = 0, dz = 0;
  if (px < bmin[0] || px > bmax[0]) {
    float d1 = std::fabs(px - bmin[0]), d2 = std::fabs(px - bmax[0]);
    dx = d1 < d2 ? d1 : d2;
  }
  if (py < bmin[1] || py > bmax[1]) {
    float d1 = std::fabs(py - bmin[1]), d2 = std::fabs(py - bmax[1]);
    dy = d1 < d2 ? d1 : d2;
  }
  if (pz < bmin[2] || pz > bmax[2]) {
    float d1 = std::fabs(pz - bmin[2]), d2 = std::fabs(pz - bmax[2]);
    dz = d1 < d2 ? d1 : d2;
  }
  return dx * dx + dy * dy + dz * dz;
}
inline void push3(float d, float& b0, float& b1, float& b2) {
  if (d < b0) { b2 = b1; b1 = b0; b0 = d; }
  else if (d < b1) { b2 = b1; b1 = d; }
  else if (d < b2) { b2 = d; }
}
}  // namespace

// Global bounds with the degenerate-extent widening of knn.py:303-315
// (done in double, then rounded to float32 like the wp.float32 kernel args).
OR_EXPORT void or_knn_bounds(int P, const float* pts, float* mn, float* mx) {
  float lo[3] = {pts[0], pts[1], pts[2]}, hi[3] = {pts[0], pts[1], pts[2]};
  for (int i = 1; i < P; ++i)
    for (int a = 0; a < 3; ++a) {
      float v = pts[i * 3 + a];
      if (v < lo[a]) lo[a] = v;
      if (v > hi[a]) hi[a] = v;
    }
  for (int a = 0; a < 3; ++a) {
    double l = lo[a], h = hi[a];
    if (h - l < 1e-7) h = l + 1e-7;
    mn[a] = (float)l;
    mx[a] = (float)h;
  }
}

OR_EXPORT void or_knn_codes(int P, const float* pts, const float* mn, const float* mx,
                            uint32_t* codes) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; ++i) {
    const float* p = pts + i * 3;
    uint32_t nx = f2u((p[0] - mn[0]) / (mx[0] - mn[0]) * 1023.0f);
    uint32_t ny = f2u((p[1] - mn[1]) / (mx[1] - mn[1]) * 1023.0f);
    uint32_t nz = f2u((p[2] - mn[2]) / (mx[2] - mn[2]) * 1023.0f);
    codes[i] = prep_morton(nx) | (prep_morton(ny) << 1) | (prep_morton(nz) << 2);
  }
}

// Returns the number of candidate distance evaluations (for the work count).
OR_EXPORT long long or_knn(int P, const float* pts, float* out) {
  if (P < 4) return -1;
  float mn[3], mx[3];
  or_knn_bounds(P, pts, mn, mx);
  std::vector<uint32_t> codes(P);
  or_knn_codes(P, pts, mn, mx, codes.data());
  std::vector<int> order(P);
  for (int i = 0; i < P; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return codes[a] < codes[b]; });
  std::vector<float> sx(P), sy(P), sz(P);
  for (int i = 0; i < P; ++i) {
    sx[i] = pts[order[i] * 3];
    sy[i] = pts[order[i] * 3 + 1];
    sz[i] = pts[order[i] * 3 + 2];
  }
  const int nb = (P + 1023) / 1024;
  std::vector<float> bmin((size_t)nb * 3), bmax((size_t)nb * 3);
  for (int b = 0; b < nb; ++b) {
    float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int i = b * 1024; i < std::min(P, (b + 1) * 1024); ++i) {
      float v[3] = {sx[i], sy[i], sz[i]};
      for (int a = 0; a < 3; ++a) {
        if (v[a] < lo[a]) lo[a] = v[a];
        if (v[a] > hi[a]) hi[a] = v[a];
      }
    }
    for (int a = 0; a < 3; ++a) { bmin[b * 3 + a] = lo[a]; bmax[b * 3 + a] = hi[a]; }
  }
  long long evals = 0;
#pragma omp parallel for schedule(dynamic, 256) reduction(+ : evals)
  for (int idx = 0; idx < P; ++idx) {
    float px = sx[idx], py = sy[idx], pz = sz[idx];
    float b0 = FLT_BIG, b1 = FLT_BIG, b2 = FLT_BIG;
    int lo = std::max(0, idx - 3), hi = std::min(P - 1, idx + 3);
    for (int i = lo; i <= hi; ++i) {
      if (i == idx) continue;
      float dx = px - sx[i], dy = py - sy[i], dz = pz - sz[i];
      push3(dx * dx + dy * dy + dz * dz, b0, b1, b2);
    }
    float reject = b2;
    b0 = b1 = b2 = FLT_BIG;
    for (int b = 0; b < nb; ++b) {
      float bd = box_dist(&bmin[b * 3], &bmax[b * 3], px, py, pz);
      if (bd > reject || bd > b2) continue;
      int e = std::min(P, (b + 1) * 1024);
      for (int i = b * 1024; i < e; ++i) {
        if (i == idx) continue;
        float dx = px - sx[i], dy = py - sy[i], dz = pz - sz[i];
        push3(dx * dx + dy * dy + dz * dz, b0, b1, b2);
      }
      evals += e - b * 1024;
    }
    out[order[idx]] = (b0 + b1 + b2) / 3.0f;
  }
  return evals;
}

// Exhaustive O(P^2) 3-NN with the same distance expression (small P only).
OR_EXPORT void or_knn_bruteforce(int P, const float* pts, float* out) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; ++i) {
    float b0 = FLT_BIG, b1 = FLT_BIG, b2 = FLT_BIG;
    for (int j = 0; j < P; ++j) {
      if (j == i) continue;
      float dx = pts[i * 3] - pts[j * 3], dy = pts[i * 3 + 1] - pts[j * 3 + 1],
            dz = pts[i * 3 + 2] - pts[j * 3 + 2];
      push3(dx * dx + dy * dy + dz * dz, b0, b1, b2);
    }
    out[i] = (b0 + b1 + b2) / 3.0f;
  }
}

OR_EXPORT int or_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// Thread count of the following parallel regions (overrides OMP_NUM_THREADS,
// which launchers such as torchrun set to 1).
OR_EXPORT void or_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
