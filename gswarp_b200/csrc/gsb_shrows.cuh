// gsb_shrows.cuh -- warp-cooperative moves of SH rows between global and
// shared memory (sm_100a).
//
// A warp handles 32 consecutive Gaussians, whose SH rows (RF = K*3 floats
// each) form one contiguous span of 32*RF floats.  Moving that span with
// lane-strided accesses is fully coalesced, where one thread per row would
// issue 32 accesses RF floats apart.  Rows land in shared memory with a
// stride of ROWF floats (odd, so that per-thread scalar accesses of a warp
// hit 32 different banks).  Only rows whose bit is set in `mask` move.
#pragma once

#include "gsb_common.cuh"

namespace gsb {

// global -> shared.  K = 16 rows (48 floats, 16-byte aligned span) move as
// float4; other widths as floats, the (row, element) index advanced without
// a division.
template <int ROWF>
__device__ __forceinline__ void sh_rows_load(float* rows, const float* src, int RF, int nrows, unsigned mask,
                                             int lane) {
  if (RF == 48 && !(reinterpret_cast<uintptr_t>(src) & 15)) {
    // 12 float4 per row, 32 rows: exactly 12 per lane, all loads issued first
    const float4* s4 = reinterpret_cast<const float4*>(src);
    const int n = nrows * 12;
    float4 v[12];
#pragma unroll
    for (int it = 0; it < 12; ++it) {
      const int j = lane + 32 * it;
      const int r = j / 12;
      v[it] = (j < n && ((mask >> r) & 1u)) ? __ldg(s4 + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int it = 0; it < 12; ++it) {
      const int j = lane + 32 * it;
      const int r = j / 12, q = j - r * 12;
      if (j < n && ((mask >> r) & 1u)) {
        float* d = rows + r * ROWF + q * 4;
        d[0] = v[it].x;
        d[1] = v[it].y;
        d[2] = v[it].z;
        d[3] = v[it].w;
      }
    }
    return;
  }
  const int n = nrows * RF;
  int r = 0, e = lane;
  while (e >= RF) {
    e -= RF;
    ++r;
  }
  for (int j = lane; j < n; j += 32) {
    if ((mask >> r) & 1u) rows[r * ROWF + e] = __ldg(src + j);
    e += 32;
    while (e >= RF) {
      e -= RF;
      ++r;
    }
  }
}

// shared -> global: dst = row (store), or dst += row (add) for the rows in
// `mask`; rows outside `mask` are stored as zero when zero_others is set.
template <int ROWF>
__device__ __forceinline__ void sh_rows_store(float* dst, const float* rows, int RF, int nrows, unsigned mask,
                                              bool add, bool zero_others, int lane) {
  if (RF == 48 && !(reinterpret_cast<uintptr_t>(dst) & 15)) {
    float4* d4 = reinterpret_cast<float4*>(dst);
    const int n = nrows * 12;
#pragma unroll 4
    for (int j = lane; j < n; j += 32) {
      const int r = j / 12, q = j - r * 12;
      const bool in = (mask >> r) & 1u;
      if (!in && !zero_others) continue;
      float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (in) {
        const float* sr = rows + r * ROWF + q * 4;
        v = make_float4(sr[0], sr[1], sr[2], sr[3]);
        if (add) {
          const float4 o = d4[j];
          v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
        }
      }
      d4[j] = v;
    }
    return;
  }
  const int n = nrows * RF;
  int r = 0, e = lane;
  while (e >= RF) {
    e -= RF;
    ++r;
  }
  for (int j = lane; j < n; j += 32) {
    const bool in = (mask >> r) & 1u;
    if (in)
      dst[j] = add ? dst[j] + rows[r * ROWF + e] : rows[r * ROWF + e];
    else if (zero_others)
      dst[j] = 0.0f;
    e += 32;
    while (e >= RF) {
      e -= RF;
      ++r;
    }
  }
}

}  // namespace gsb
