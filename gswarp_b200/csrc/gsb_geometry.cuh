// gsb_geometry.cuh -- screen-space footprint and AccuTile tile coverage.
//
// Device restatement of gswarp's math_kernels.py:86-390 and the emission
// loops of binning_kernels.py:126-216.  Every translation unit that includes
// this header is compiled with -fmad=false (no FMA contraction), IEEE
// division and square root, so the tile counts computed in preprocess and
// the tiles emitted during binning are bit-identical to each other and to
// the CPU oracle; the count/emit agreement is what keeps the pair buffer
// exactly filled.
#pragma once

#include "gsb_common.cuh"

namespace gsb {

constexpr float DET_EPSILON = 1.0e-7f;
constexpr float SNUGBOX_PIXEL_PADDING = 1.0f;
constexpr float COVERAGE_Q_EPSILON = 1.0e-4f;
constexpr float FLT_BIG = 3.402823466e38f;

struct Rect {
  int x0, y0, x1, y1;
};

// math_kernels.py:86-87
__device__ __forceinline__ float ndc2pix(float v, int size) {
  return ((v + 1.0f) * (float)size - 1.0f) * 0.5f;
}

// math_kernels.py:136-148 (CUDA getRect)
__device__ __forceinline__ Rect tile_rect(float px, float py, int radius, int gx, int gy) {
  Rect r;
  r.x0 = imn(gx, imx(0, f2i((px - (float)radius) / (float)BLOCK_X)));
  r.y0 = imn(gy, imx(0, f2i((py - (float)radius) / (float)BLOCK_Y)));
  r.x1 = imn(gx, imx(0, f2i((px + (float)radius + (float)(BLOCK_X - 1)) / (float)BLOCK_X)));
  r.y1 = imn(gy, imx(0, f2i((py + (float)radius + (float)(BLOCK_Y - 1)) / (float)BLOCK_Y)));
  return r;
}

// Opacity threshold 2*ln(max(255*op, 1)) of math_kernels.py:170,340.
__device__ __forceinline__ float opacity_threshold(float opacity) {
  return 2.0f * crlogf(fmx(255.0f * opacity, 1.0f));
}

// math_kernels.py:150-194: padded SnugBox clipped to the CUDA 3-sigma rect.
__device__ __forceinline__ Rect snugbox_rect(float px, float py, float cov_aa, float cov_cc,
                                             float t, int cuda_radius, int gx, int gy) {
  Rect c = tile_rect(px, py, cuda_radius, gx, gy);
  if (t <= 0.0f) return Rect{0, 0, 0, 0};
  int rx = f2i(ceilf(sqrtf(fmx(t * cov_aa, 0.0f)) + SNUGBOX_PIXEL_PADDING));
  int ry = f2i(ceilf(sqrtf(fmx(t * cov_cc, 0.0f)) + SNUGBOX_PIXEL_PADDING));
  Rect s;
  s.x0 = imn(gx, imx(0, f2i((px - (float)rx) / (float)BLOCK_X)));
  s.y0 = imn(gy, imx(0, f2i((py - (float)ry) / (float)BLOCK_Y)));
  s.x1 = imn(gx, imx(0, f2i((px + (float)rx + (float)(BLOCK_X - 1)) / (float)BLOCK_X)));
  s.y1 = imn(gy, imx(0, f2i((py + (float)ry + (float)(BLOCK_Y - 1)) / (float)BLOCK_Y)));
  return Rect{imx(c.x0, s.x0), imx(c.y0, s.y0), imn(c.x1, s.x1), imn(c.y1, s.y1)};
}

// math_kernels.py:196-204
__device__ __forceinline__ float conic_q(float x, float y, float a, float b, float c) {
  return a * x * x + 2.0f * b * x * y + c * y * y;
}

// math_kernels.py:206-240
__device__ __forceinline__ bool conic_rect_intersects(float px, float py, float a, float b,
                                                      float c, float threshold, int tx, int ty) {
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

// math_kernels.py:242-303: AccuTile tile interval of one band.  The terms
// that do not depend on the band (determinant, padded threshold, the
// ellipse's u-extent and the v at its u-extremes) are computed once per
// Gaussian by band_setup, with the same expressions, so every band sees the
// same bits as a per-band evaluation.
struct BandSetup {
  bool degenerate;
  float det, ts, extent_u, v_at_min_u, v_at_max_u;
};

__device__ __forceinline__ BandSetup band_setup(float cuu, float cuv, float cvv, float threshold) {
  BandSetup b;
  b.det = cuu * cvv - cuv * cuv;
  b.degenerate = cuu <= 0.0f || cvv <= 0.0f || b.det <= DET_EPSILON;
  b.ts = threshold + COVERAGE_Q_EPSILON;
  // unused (and possibly not finite) when degenerate
  b.extent_u = sqrtf(fmx(b.ts * cvv / b.det, 0.0f));
  b.v_at_min_u = cuv * b.extent_u / cvv;
  b.v_at_max_u = -cuv * b.extent_u / cvv;
  return b;
}

__device__ __forceinline__ void band_interval(float pu, float pv, float cuu, float cuv, const BandSetup& bs,
                                              int tile_v, int block_u, int block_v, int rect_u_min,
                                              int rect_u_max, int& lo, int& hi) {
  if (bs.degenerate) {
    lo = rect_u_min;
    hi = rect_u_max;
    return;
  }
  const float det = bs.det, ts = bs.ts;
  float v0 = (float)(tile_v * block_v) - pv;
  float v1 = (float)(tile_v * block_v + block_v - 1) - pv;
  float u_min = FLT_BIG, u_max = -FLT_BIG;
  bool found = false;
  float disc = cuu * ts - det * v0 * v0;
  if (disc >= -COVERAGE_Q_EPSILON) {
    float half = sqrtf(fmx(disc, 0.0f)) / cuu;
    float center = -cuv * v0 / cuu;
    u_min = fmn(u_min, center - half);
    u_max = fmx(u_max, center + half);
    found = true;
  }
  disc = cuu * ts - det * v1 * v1;
  if (disc >= -COVERAGE_Q_EPSILON) {
    float half = sqrtf(fmx(disc, 0.0f)) / cuu;
    float center = -cuv * v1 / cuu;
    u_min = fmn(u_min, center - half);
    u_max = fmx(u_max, center + half);
    found = true;
  }
  const float extent_u = bs.extent_u;
  if (bs.v_at_min_u >= v0 - COVERAGE_Q_EPSILON && bs.v_at_min_u <= v1 + COVERAGE_Q_EPSILON) {
    u_min = fmn(u_min, -extent_u);
    u_max = fmx(u_max, -extent_u);
    found = true;
  }
  if (bs.v_at_max_u >= v0 - COVERAGE_Q_EPSILON && bs.v_at_max_u <= v1 + COVERAGE_Q_EPSILON) {
    u_min = fmn(u_min, extent_u);
    u_max = fmx(u_max, extent_u);
    found = true;
  }
  if (!found) {
    lo = rect_u_min;
    hi = rect_u_min;
    return;
  }
  int tmin = f2i(floorf((pu + u_min) / (float)block_u));
  int tmax = f2i(floorf((pu + u_max) / (float)block_u)) + 1;
  lo = imx(rect_u_min, imn(rect_u_max, tmin));
  hi = imx(rect_u_min, imn(rect_u_max, tmax));
}

// Tile coverage of one Gaussian (math_kernels.py:305-390; conic_rect as
// recounted by binning_kernels.py:56-124).  With EMIT=true
// it also writes every covered tile id, in the reference's emission order
// (binning_kernels.py:141-216), through emit(tile_id).
struct NoEmit {
  __device__ __forceinline__ void operator()(int) const {}
};

// The two halves of cover_tiles: the footprint's opacity threshold and
// clipped SnugBox rect (which need the 2D covariance and the radius), then
// the tile sweep inside the rect (which needs only the centre, the conic and
// the threshold).  Preprocess stores (rect, threshold) per Gaussian so the
// binning emit can run the second half alone, on the same bits.
__device__ __forceinline__ void coverage_setup(float px, float py, float cov_aa, float cov_cc,
                                               float opacity, int cuda_radius, int gx, int gy,
                                               Rect& r, float& t) {
  t = opacity_threshold(opacity);
  r = snugbox_rect(px, py, cov_aa, cov_cc, t, cuda_radius, gx, gy);
}

template <typename Emit>
__device__ __forceinline__ int cover_tiles_in_rect(float px, float py, float ca, float cb, float cc,
                                                   float t, const Rect r, int gx, int mode,
                                                   const Emit& emit) {
  int span_x = r.x1 - r.x0;
  int span_y = r.y1 - r.y0;
  int area = span_x * span_y;
  if (area <= 1 || mode == GSB_COVERAGE_SNUGBOX) {
    for (int ty = r.y0; ty < r.y1; ++ty)
      for (int tx = r.x0; tx < r.x1; ++tx) emit(ty * gx + tx);
    return area;
  }
  int count = 0;
  // conic_rect keeps its per-tile test only for footprints of at most 64
  // tiles and falls back to the AccuTile sweep above that, which is what the
  // reference's binning recount applies (binning_kernels.py:56-124).
  if (mode == GSB_COVERAGE_CONIC_RECT && area <= 64) {
    for (int ty = r.y0; ty < r.y1; ++ty)
      for (int tx = r.x0; tx < r.x1; ++tx)
        if (conic_rect_intersects(px, py, ca, cb, cc, t, tx, ty)) {
          ++count;
          emit(ty * gx + tx);
        }
    return count;
  }
  if (span_y <= span_x) {
    const BandSetup bs = band_setup(ca, cb, cc, t);
    for (int ty = r.y0; ty < r.y1; ++ty) {
      int lo, hi;
      band_interval(px, py, ca, cb, bs, ty, BLOCK_X, BLOCK_Y, r.x0, r.x1, lo, hi);
      count += imx(0, hi - lo);
      for (int tx = lo; tx < hi; ++tx) emit(ty * gx + tx);
    }
  } else {
    const BandSetup bs = band_setup(cc, cb, ca, t);
    for (int tx = r.x0; tx < r.x1; ++tx) {
      int lo, hi;
      band_interval(py, px, cc, cb, bs, tx, BLOCK_Y, BLOCK_X, r.y0, r.y1, lo, hi);
      count += imx(0, hi - lo);
      for (int ty = lo; ty < hi; ++ty) emit(ty * gx + tx);
    }
  }
  return count;
}

template <typename Emit>
__device__ __forceinline__ int cover_tiles(float px, float py, float cov_aa, float cov_cc,
                                           float ca, float cb, float cc, float opacity,
                                           int cuda_radius, int gx, int gy, int mode,
                                           const Emit& emit) {
  Rect r;
  float t;
  coverage_setup(px, py, cov_aa, cov_cc, opacity, cuda_radius, gx, gy, r, t);
  return cover_tiles_in_rect(px, py, ca, cb, cc, t, r, gx, mode, emit);
}

// 32-byte binning record of a Gaussian with tiles, written by preprocess
// while it counts the tiles, so that the binning emit only replays the
// result: words 0-1 hold the clipped rect (x0 | y0 << 16, x1 | y1 << 16;
// tile grids below 65536), word 2 the kind (bits 0-1), the band direction
// (bit 2: bands are tile columns) and the band count (bits 8-15), words 3-7
// the payload:
//   BINREC_RECT  every tile of the rect (area <= 1, or SnugBox mode);
//   BINREC_BANDS the AccuTile [lo, hi) of each band, lo | hi << 16, up to 5;
//   BINREC_MASK  conic_rect per-tile results for rects of <= 64 tiles,
//                row-major bits in words 3-4;
//   BINREC_SWEEP more than 5 bands: the emit re-runs the sweep from the
//                render record (same inputs, same bits).
constexpr unsigned BINREC_RECT = 0, BINREC_BANDS = 1, BINREC_MASK = 2, BINREC_SWEEP = 3;
constexpr int BINREC_MAX_BANDS = 5;

// Counts the tiles of cover_tiles_in_rect and fills the record; the count
// is the one cover_tiles_in_rect returns (same calls, same order).
__device__ __forceinline__ int coverage_record(float px, float py, float ca, float cb, float cc, float t,
                                               const Rect r, int mode, unsigned (&w)[8]) {
  w[0] = (unsigned)r.x0 | ((unsigned)r.y0 << 16);
  w[1] = (unsigned)r.x1 | ((unsigned)r.y1 << 16);
  w[2] = w[3] = w[4] = w[5] = w[6] = w[7] = 0u;
  const int span_x = r.x1 - r.x0, span_y = r.y1 - r.y0;
  const int area = span_x * span_y;
  if (area <= 1 || mode == GSB_COVERAGE_SNUGBOX) {
    w[2] = BINREC_RECT;
    return area;
  }
  int count = 0;
  if (mode == GSB_COVERAGE_CONIC_RECT && area <= 64) {
    unsigned long long mask = 0ull;
    int bit = 0;
    for (int ty = r.y0; ty < r.y1; ++ty)
      for (int tx = r.x0; tx < r.x1; ++tx, ++bit)
        if (conic_rect_intersects(px, py, ca, cb, cc, t, tx, ty)) {
          ++count;
          mask |= 1ull << bit;
        }
    w[2] = BINREC_MASK;
    w[3] = (unsigned)mask;
    w[4] = (unsigned)(mask >> 32);
    return count;
  }
  const bool vertical = span_y > span_x;
  const int nb = vertical ? span_x : span_y;
  const bool fits = nb <= BINREC_MAX_BANDS;
  w[2] = (fits ? BINREC_BANDS : BINREC_SWEEP) | (vertical ? 4u : 0u) | ((unsigned)nb << 8);
  const BandSetup bs = vertical ? band_setup(cc, cb, ca, t) : band_setup(ca, cb, cc, t);
  for (int b = 0; b < nb; ++b) {
    int lo, hi;
    if (!vertical)
      band_interval(px, py, ca, cb, bs, r.y0 + b, BLOCK_X, BLOCK_Y, r.x0, r.x1, lo, hi);
    else
      band_interval(py, px, cc, cb, bs, r.x0 + b, BLOCK_Y, BLOCK_X, r.y0, r.y1, lo, hi);
    count += imx(0, hi - lo);
    if (fits && b < BINREC_MAX_BANDS) w[3 + b] = (unsigned)lo | ((unsigned)hi << 16);
  }
  return count;
}

// Emits the tiles of a binning record in cover_tiles_in_rect's order.
// BINREC_SWEEP records need the sweep inputs, passed in by the caller.
template <typename Emit>
__device__ __forceinline__ void emit_record(const unsigned (&w)[8], int gx, int mode, float px, float py, float ca,
                                            float cb, float cc, float t, const Emit& emit) {
  Rect r;
  r.x0 = (int)(w[0] & 0xFFFFu);
  r.y0 = (int)(w[0] >> 16);
  r.x1 = (int)(w[1] & 0xFFFFu);
  r.y1 = (int)(w[1] >> 16);
  const unsigned kind = w[2] & 3u;
  const bool vertical = (w[2] >> 2) & 1u;
  const int nb = (int)((w[2] >> 8) & 0xFFu);
  if (kind == BINREC_RECT) {
    for (int ty = r.y0; ty < r.y1; ++ty)
      for (int tx = r.x0; tx < r.x1; ++tx) emit(ty * gx + tx);
  } else if (kind == BINREC_MASK) {
    const unsigned long long mask = (unsigned long long)w[3] | ((unsigned long long)w[4] << 32);
    int bit = 0;
    for (int ty = r.y0; ty < r.y1; ++ty)
      for (int tx = r.x0; tx < r.x1; ++tx, ++bit)
        if ((mask >> bit) & 1ull) emit(ty * gx + tx);
  } else if (kind == BINREC_BANDS) {
#pragma unroll 1
    for (int b = 0; b < nb; ++b) {
      const int lo = (int)(w[3 + b] & 0xFFFFu), hi = (int)(w[3 + b] >> 16);
      if (!vertical)
        for (int tx = lo; tx < hi; ++tx) emit((r.y0 + b) * gx + tx);
      else
        for (int ty = lo; ty < hi; ++ty) emit(ty * gx + r.x0 + b);
    }
  } else {
    cover_tiles_in_rect(px, py, ca, cb, cc, t, r, gx, mode, emit);
  }
}

}  // namespace gsb
