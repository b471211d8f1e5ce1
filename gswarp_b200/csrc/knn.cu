// knn.cu -- Morton-ordered, box-pruned exact 3-nearest-neighbour distances.
//
// Restates gswarp's distCUDA2 (knn.py:264-401): global AABB with the 1e-7
// degenerate-extent widening (done here on the device in fp64, without the
// reference's six .item() host syncs), 30-bit Morton codes (:48-67,
// :108-119), stable radix sort of (code, index) (:334-341), gather into
// sorted SoA, per-1024-point box AABBs (:137-162) and the box-pruned 3-NN
// search seeded from the +-3 sorted neighbours (:165-256).
//
// The pruning is exact (a box is skipped only when its lower-bound distance
// exceeds the current third-best), so the result is the mean of the three
// smallest squared distances whatever order boxes are visited in; this
// kernel visits the point's own box first, which tightens the bound early.
// Built with -fmad=false so distances match the CPU oracle bit for bit.
//
// B200 layout: box AABBs are computed with one CTA per box (block min/max
// reductions instead of the reference's 6 float atomics per point) and are
// staged in shared memory by every search CTA (24 bytes per box: up to 9,000
// boxes = 9.2M points fit in 227 KB; larger inputs read them from L2).
#include <algorithm>

#include "gsb_common.cuh"
#include "radix_sort.cuh"

namespace gsb {
namespace {

constexpr int BOX = 1024;
constexpr int BOUNDS_BLOCKS = 296;
constexpr float FLT_BIG_K = 3.402823466e38f;

__global__ void __launch_bounds__(256) bounds_partial_kernel(int P, const float* __restrict__ pts,
                                                             float* __restrict__ part) {
  float lo[3] = {FLT_BIG_K, FLT_BIG_K, FLT_BIG_K}, hi[3] = {-FLT_BIG_K, -FLT_BIG_K, -FLT_BIG_K};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P; i += gridDim.x * blockDim.x) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float v = pts[(size_t)i * 3 + c];
      lo[c] = fminf(lo[c], v);
      hi[c] = fmaxf(hi[c], v);
    }
  }
  __shared__ float s[6][8];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo[c] = fminf(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
      hi[c] = fmaxf(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
    }
  }
  if ((threadIdx.x & 31) == 0)
    for (int c = 0; c < 3; ++c) {
      s[c][threadIdx.x >> 5] = lo[c];
      s[3 + c][threadIdx.x >> 5] = hi[c];
    }
  __syncthreads();
  if (threadIdx.x < 6) {
    float r = s[threadIdx.x][0];
    for (int w = 1; w < 8; ++w)
      r = threadIdx.x < 3 ? fminf(r, s[threadIdx.x][w]) : fmaxf(r, s[threadIdx.x][w]);
    part[blockIdx.x * 6 + threadIdx.x] = r;
  }
}

// knn.py:304-315: min/max, then widen degenerate extents in double precision
// and round to float32 like the reference's wp.float32(...) kernel arguments.
__global__ void bounds_final_kernel(int nparts, const float* __restrict__ part,
                                    float* __restrict__ bounds) {
  if (threadIdx.x != 0) return;
  float lo[3], hi[3];
  for (int c = 0; c < 3; ++c) {
    lo[c] = part[c];
    hi[c] = part[3 + c];
  }
  for (int b = 1; b < nparts; ++b)
    for (int c = 0; c < 3; ++c) {
      lo[c] = fminf(lo[c], part[b * 6 + c]);
      hi[c] = fmaxf(hi[c], part[b * 6 + 3 + c]);
    }
  for (int c = 0; c < 3; ++c) {
    const double l = lo[c];
    double h = hi[c];
    if (h - l < 1e-7) h = l + 1e-7;
    bounds[c] = (float)l;
    bounds[3 + c] = (float)h;
  }
}

__device__ __forceinline__ unsigned prep_morton(unsigned x) {
  x = (x | (x << 16)) & 0x030000FFu;
  x = (x | (x << 8)) & 0x0300F00Fu;
  x = (x | (x << 4)) & 0x030C30C3u;
  x = (x | (x << 2)) & 0x09249249u;
  return x;
}

__global__ void morton_kernel(int P, const float* __restrict__ pts,
                              const float* __restrict__ bounds, unsigned* __restrict__ codes,
                              unsigned* __restrict__ idx) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const float mnx = bounds[0], mny = bounds[1], mnz = bounds[2];
  const float mxx = bounds[3], mxy = bounds[4], mxz = bounds[5];
  const float x = pts[(size_t)i * 3], y = pts[(size_t)i * 3 + 1], z = pts[(size_t)i * 3 + 2];
  const unsigned nx = __float2uint_rz((x - mnx) / (mxx - mnx) * 1023.0f);
  const unsigned ny = __float2uint_rz((y - mny) / (mxy - mny) * 1023.0f);
  const unsigned nz = __float2uint_rz((z - mnz) / (mxz - mnz) * 1023.0f);
  codes[i] = prep_morton(nx) | (prep_morton(ny) << 1) | (prep_morton(nz) << 2);
  idx[i] = (unsigned)i;
}

// One CTA per 1024-point box: gather sorted SoA and the box AABB.
__global__ void __launch_bounds__(256) gather_box_kernel(int P, const float* __restrict__ pts,
                                                         const unsigned* __restrict__ order,
                                                         float* __restrict__ sx,
                                                         float* __restrict__ sy,
                                                         float* __restrict__ sz,
                                                         float* __restrict__ boxes) {
  const int b = blockIdx.x;
  float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
  for (int k = threadIdx.x; k < BOX; k += 256) {
    const int i = b * BOX + k;
    if (i >= P) break;
    const unsigned o = order[i];
    const float v[3] = {pts[(size_t)o * 3], pts[(size_t)o * 3 + 1], pts[(size_t)o * 3 + 2]};
    sx[i] = v[0];
    sy[i] = v[1];
    sz[i] = v[2];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      lo[c] = fminf(lo[c], v[c]);
      hi[c] = fmaxf(hi[c], v[c]);
    }
  }
  __shared__ float s[6][8];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo[c] = fminf(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
      hi[c] = fmaxf(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
    }
  }
  if ((threadIdx.x & 31) == 0)
    for (int c = 0; c < 3; ++c) {
      s[c][threadIdx.x >> 5] = lo[c];
      s[3 + c][threadIdx.x >> 5] = hi[c];
    }
  __syncthreads();
  if (threadIdx.x < 6) {
    float r = s[threadIdx.x][0];
    for (int w = 1; w < 8; ++w)
      r = threadIdx.x < 3 ? fminf(r, s[threadIdx.x][w]) : fmaxf(r, s[threadIdx.x][w]);
    boxes[(size_t)b * 6 + threadIdx.x] = r;  // minx,miny,minz,maxx,maxy,maxz
  }
}

// knn.py:71-100
__device__ __forceinline__ float box_dist(const float* bx, float px, float py, float pz) {
  float dx = 0.0f, dy = 0.0f, dz = 0.0f;
  if (px < bx[0] || px > bx[3]) {
    const float d1 = fabsf(px - bx[0]), d2 = fabsf(px - bx[3]);
    dx = d1 < d2 ? d1 : d2;
  }
  if (py < bx[1] || py > bx[4]) {
    const float d1 = fabsf(py - bx[1]), d2 = fabsf(py - bx[4]);
    dy = d1 < d2 ? d1 : d2;
  }
  if (pz < bx[2] || pz > bx[5]) {
    const float d1 = fabsf(pz - bx[2]), d2 = fabsf(pz - bx[5]);
    dz = d1 < d2 ? d1 : d2;
  }
  return dx * dx + dy * dy + dz * dz;
}

__device__ __forceinline__ void push3(float d, float& b0, float& b1, float& b2) {
  if (d < b0) {
    b2 = b1;
    b1 = b0;
    b0 = d;
  } else if (d < b1) {
    b2 = b1;
    b1 = d;
  } else if (d < b2) {
    b2 = d;
  }
}

__device__ __forceinline__ void scan_box(int b, int P, int idx, float px, float py, float pz,
                                         const float* __restrict__ sx, const float* __restrict__ sy,
                                         const float* __restrict__ sz, float& b0, float& b1,
                                         float& b2) {
  const int e = min(P, (b + 1) * BOX);
  for (int i = b * BOX; i < e; ++i) {
    if (i == idx) continue;
    const float dx = px - __ldg(sx + i), dy = py - __ldg(sy + i), dz = pz - __ldg(sz + i);
    push3(dx * dx + dy * dy + dz * dz, b0, b1, b2);
  }
}

template <bool SMEM_BOXES>
__global__ void __launch_bounds__(256) search_kernel(int P, int nb, const float* __restrict__ sx,
                                                     const float* __restrict__ sy,
                                                     const float* __restrict__ sz,
                                                     const float* __restrict__ boxes_g,
                                                     const unsigned* __restrict__ order,
                                                     float* __restrict__ out) {
  extern __shared__ float s_boxes[];
  const float* boxes = boxes_g;
  if (SMEM_BOXES) {
    for (int i = threadIdx.x; i < nb * 6; i += blockDim.x) s_boxes[i] = boxes_g[i];
    __syncthreads();
    boxes = s_boxes;
  }
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= P) return;
  const float px = sx[idx], py = sy[idx], pz = sz[idx];
  float b0 = FLT_BIG_K, b1 = FLT_BIG_K, b2 = FLT_BIG_K;
  const int lo = max(0, idx - 3), hi = min(P - 1, idx + 3);
  for (int i = lo; i <= hi; ++i) {
    if (i == idx) continue;
    const float dx = px - sx[i], dy = py - sy[i], dz = pz - sz[i];
    push3(dx * dx + dy * dy + dz * dz, b0, b1, b2);
  }
  const float reject = b2;
  b0 = b1 = b2 = FLT_BIG_K;
  const int own = idx / BOX;
  {
    const float bd = box_dist(boxes + own * 6, px, py, pz);
    if (!(bd > reject || bd > b2)) scan_box(own, P, idx, px, py, pz, sx, sy, sz, b0, b1, b2);
  }
  for (int b = 0; b < nb; ++b) {
    if (b == own) continue;
    const float bd = box_dist(boxes + b * 6, px, py, pz);
    if (bd > reject || bd > b2) continue;
    scan_box(b, P, idx, px, py, pz, sx, sy, sz, b0, b1, b2);
  }
  out[order[idx]] = (b0 + b1 + b2) / 3.0f;
}

inline size_t a256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT size_t gsb_knn_workspace_bytes(int P) {
  const size_t n = (size_t)(P > 0 ? P : 1);
  const size_t nb = (n + BOX - 1) / BOX;
  size_t b = a256(n * 4) * 4;        // codes, codes_alt, idx, idx_alt
  b += a256(n * 4) * 3;              // sx, sy, sz
  b += a256(nb * 6 * 4);             // boxes
  b += a256((size_t)BOUNDS_BLOCKS * 6 * 4) + 256;  // partials + bounds
  b += radix::scratch_bytes((long long)n, 4);
  return b + 256;
}

GSB_EXPORT int gsb_knn(const gsb_knn_args* a, void* stream) {
  if (!a || a->P < 4 || !a->points || !a->out || !a->error_word || !a->workspace ||
      a->workspace_bytes < gsb_knn_workspace_bytes(a->P)) {
    set_error("gsb_knn: invalid arguments (P >= 4, pointers, workspace size)");
    return GSB_ERR_INVALID;
  }
  const int P = a->P;
  const int nb = (P + BOX - 1) / BOX;
  cudaStream_t s = (cudaStream_t)stream;
  char* w = (char*)(((uintptr_t)a->workspace + 255) & ~(uintptr_t)255);
  auto take = [&](size_t bytes) {
    char* p = w;
    w += a256(bytes);
    return p;
  };
  unsigned* codes = (unsigned*)take((size_t)P * 4);
  unsigned* codes_alt = (unsigned*)take((size_t)P * 4);
  unsigned* idx = (unsigned*)take((size_t)P * 4);
  unsigned* idx_alt = (unsigned*)take((size_t)P * 4);
  float* sx = (float*)take((size_t)P * 4);
  float* sy = (float*)take((size_t)P * 4);
  float* sz = (float*)take((size_t)P * 4);
  float* boxes = (float*)take((size_t)nb * 6 * 4);
  float* part = (float*)take((size_t)BOUNDS_BLOCKS * 6 * 4);
  float* bounds = (float*)take(256);
  void* scratch = w;

  bounds_partial_kernel<<<BOUNDS_BLOCKS, 256, 0, s>>>(P, a->points, part);
  bounds_final_kernel<<<1, 32, 0, s>>>(BOUNDS_BLOCKS, part, bounds);
  morton_kernel<<<div_up(P, 256), 256, 0, s>>>(P, a->points, bounds, codes, idx);
  unsigned* kb[2] = {codes, codes_alt};
  unsigned* vb[2] = {idx, idx_alt};
  const int where = radix::sort_pairs(kb, vb, P, nullptr, 4, scratch, a->error_word, s);
  const unsigned* order = vb[where];
  gather_box_kernel<<<nb, 256, 0, s>>>(P, a->points, order, sx, sy, sz, boxes);
  const size_t smem = (size_t)nb * 6 * 4;
  if (smem <= 200 * 1024) {
    cudaFuncSetAttribute(search_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    search_kernel<true><<<div_up(P, 256), 256, smem, s>>>(P, nb, sx, sy, sz, boxes, order, a->out);
  } else {
    search_kernel<false><<<div_up(P, 256), 256, 0, s>>>(P, nb, sx, sy, sz, boxes, order, a->out);
  }
  return check_launch("gsb_knn");
}
