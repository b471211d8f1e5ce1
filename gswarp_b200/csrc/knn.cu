// knn.cu -- Morton-ordered, box-pruned exact 3-nearest-neighbour distances.
//
// Restates gswarp's distCUDA2 (knn.py:264-401): global AABB with the 1e-7
// degenerate-extent widening (done here on the device in fp64, without the
// reference's six .item() host syncs), 30-bit Morton codes (:48-67,
// :108-119), stable radix sort of (code, index) (:334-341), gather into
// sorted SoA, and a box-pruned 3-NN search (:137-256).
//
// The pruning is exact: a group of candidates is skipped only when a lower
// bound of its squared distance exceeds the current third-best, and every
// bound is computed with the same monotone float operations (no FMA
// contraction, -fmad=false) as the point distances it bounds, so the result
// is the mean of the three smallest squared distances whatever order
// candidates are visited in -- bit for bit the reference's value.
//
// B200 layout: the sorted points are grouped into leaves of 32 (one per
// lane), parents of 32 leaves (the reference's 1024-point boxes) and
// grandparents of 32 parents, each with an AABB.  One warp searches for the
// 32 consecutive sorted points of a leaf: it scans its own leaf, then walks
// grandparents -> parents -> leaves, testing 32 boxes per step (one per
// lane) against the warp's query AABB and its largest third-best, and scans
// a surviving leaf by broadcasting its 32 points with shuffles to every lane
// that still needs it (the reference instead tests every 1024-point box per
// point and scans boxes point by point).
#include <algorithm>

#include "gsb_common.cuh"
#include "radix_sort.cuh"

namespace gsb {
namespace {

constexpr int BOUNDS_BLOCKS = 296;
constexpr int KT = launch::KNN;  // threads per CTA of every KNN kernel but the final bounds reduction
constexpr float FLT_BIG_K = 3.402823466e38f;

__global__ void __launch_bounds__(KT) bounds_partial_kernel(int P, const float* __restrict__ pts,
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
  __shared__ float s[6][KT / 32];
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
    for (int w = 1; w < KT / 32; ++w)
      r = threadIdx.x < 3 ? fminf(r, s[threadIdx.x][w]) : fmaxf(r, s[threadIdx.x][w]);
    part[blockIdx.x * 6 + threadIdx.x] = r;
  }
}

// knn.py:304-315: min/max, then widen degenerate extents in double precision
// and round to float32 like the reference's wp.float32(...) kernel arguments.
__global__ void bounds_final_kernel(int nparts, const float* __restrict__ part,
                                    float* __restrict__ bounds) {
  // one warp: lanes take the partials strided, then a shuffle min/max
  // (minimum and maximum do not depend on the order)
  const int lane = threadIdx.x & 31;
  float lo[3] = {FLT_BIG_K, FLT_BIG_K, FLT_BIG_K}, hi[3] = {-FLT_BIG_K, -FLT_BIG_K, -FLT_BIG_K};
  for (int b = lane; b < nparts; b += 32)
    for (int c = 0; c < 3; ++c) {
      lo[c] = fminf(lo[c], part[b * 6 + c]);
      hi[c] = fmaxf(hi[c], part[b * 6 + 3 + c]);
    }
  for (int c = 0; c < 3; ++c)
    for (int o = 16; o > 0; o >>= 1) {
      lo[c] = fminf(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
      hi[c] = fmaxf(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
    }
  if (lane != 0) return;
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

constexpr int LEAF = 32;  // points per leaf (one per lane); 32 leaves per parent, 32 parents per grandparent

// Thread per sorted point: gather the sorted SoA; each warp (= one leaf of
// 32 consecutive sorted points) reduces its AABB.
__global__ void __launch_bounds__(KT) gather_leaf_kernel(int P, const float* __restrict__ pts,
                                                          const unsigned* __restrict__ order,
                                                          float* __restrict__ sx, float* __restrict__ sy,
                                                          float* __restrict__ sz, float* __restrict__ leaf_boxes) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int leaf = i / LEAF;
  if (leaf * LEAF >= P) return;  // whole warp past the end
  float v[3] = {0.0f, 0.0f, 0.0f};
  const bool valid = i < P;
  if (valid) {
    const unsigned o = order[i];
    v[0] = pts[(size_t)o * 3];
    v[1] = pts[(size_t)o * 3 + 1];
    v[2] = pts[(size_t)o * 3 + 2];
    sx[i] = v[0];
    sy[i] = v[1];
    sz[i] = v[2];
  }
  float lo[3], hi[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    lo[c] = valid ? v[c] : INFINITY;
    hi[c] = valid ? v[c] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo[c] = fminf(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
      hi[c] = fmaxf(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
    }
  }
  if ((threadIdx.x & 31) == 0) {
    float* b = leaf_boxes + (size_t)leaf * 6;
    b[0] = lo[0]; b[1] = lo[1]; b[2] = lo[2];
    b[3] = hi[0]; b[4] = hi[1]; b[5] = hi[2];
  }
}

// Warp per parent box: AABB of up to 32 child boxes.
__global__ void __launch_bounds__(KT) reduce_boxes_kernel(int nchild, const float* __restrict__ child,
                                                           float* __restrict__ parent) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int par = t / 32, lane = threadIdx.x & 31;
  if (par * 32 >= nchild) return;
  const int c = par * 32 + lane;
  const bool valid = c < nchild;
  float lo[3], hi[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    lo[k] = valid ? child[(size_t)c * 6 + k] : INFINITY;
    hi[k] = valid ? child[(size_t)c * 6 + 3 + k] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo[k] = fminf(lo[k], __shfl_xor_sync(0xffffffffu, lo[k], o));
      hi[k] = fmaxf(hi[k], __shfl_xor_sync(0xffffffffu, hi[k], o));
    }
  }
  if (lane == 0) {
    float* b = parent + (size_t)par * 6;
    b[0] = lo[0]; b[1] = lo[1]; b[2] = lo[2];
    b[3] = hi[0]; b[4] = hi[1]; b[5] = hi[2];
  }
}

// knn.py:71-100: squared distance from a point to an AABB (0 inside).
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

// Squared distance between two AABBs (0 when they overlap): a lower bound
// of every point-to-point distance between them, computed with the same
// rounding-monotone operations as those distances.
__device__ __forceinline__ float boxbox_dist(const float* a, const float* b) {
  float d[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    d[k] = 0.0f;
    if (a[k] > b[3 + k]) d[k] = a[k] - b[3 + k];
    else if (b[k] > a[3 + k]) d[k] = b[k] - a[3 + k];
  }
  return d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
}

// Inserts d into the sorted three smallest (b0 <= b1 <= b2): a compare-exchange
// chain, branch-free; the kept values (ties included) are the ones a
// shift-insertion keeps, in the same order.
__device__ __forceinline__ void push3(float d, float& b0, float& b1, float& b2) {
  const float c0 = fmaxf(b0, d);
  b0 = fminf(b0, d);
  const float c1 = fmaxf(b1, c0);
  b1 = fminf(b1, c0);
  b2 = fminf(b2, c1);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Candidate leaf L against every lane's query point: the warp stages the
// leaf's points in shared memory (one 16-byte slot per lane), then each lane
// reads them back by broadcast.  OWN: L is the query's own leaf, whose point
// at the lane's own position is skipped (as a +big distance, which top-3
// never keeps).
template <bool OWN>
__device__ __forceinline__ void scan_leaf(int L, int P, bool need, float px, float py, float pz,
                                          const float* __restrict__ sx, const float* __restrict__ sy,
                                          const float* __restrict__ sz, float4* s_pts, float& b0, float& b1,
                                          float& b2) {
  const int lane = threadIdx.x & 31;
  const int c = L * LEAF + lane;
  __syncwarp();  // the previous leaf's readers are done with s_pts
  s_pts[lane] = c < P ? make_float4(sx[c], sy[c], sz[c], 0.0f) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  __syncwarp();
  if (!need) return;
  const int n = min(LEAF, P - L * LEAF);
#pragma unroll 4
  for (int k = 0; k < n; ++k) {
    const float4 q = s_pts[k];
    const float dx = px - q.x, dy = py - q.y, dz = pz - q.z;
    float d = dx * dx + dy * dy + dz * dz;
    if (OWN && k == lane) d = FLT_BIG_K;
    push3(d, b0, b1, b2);
  }
}

// Candidate leaf L for the few lanes in needmask (not the query's own leaf):
// candidate-parallel instead of query-parallel.  For each needing lane q,
// every lane computes q's distance to its own candidate (same operands, same
// order as scan_leaf), three warp minimum reductions take the three smallest
// (ties kept: one lane removed per round) and q pushes them into its top
// three -- the same three smallest values as pushing all 32.  Cheaper than
// the 32-step scan when only a few lanes need the leaf (sparse regions, where
// a few far query points otherwise make the warp scan many distant leaves).
constexpr int SPARSE_LANES = 8;

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void scan_leaf_sparse(int L, int P, unsigned needmask, float px, float py, float pz,
                                                 const float* __restrict__ sx, const float* __restrict__ sy,
                                                 const float* __restrict__ sz, float& b0, float& b1, float& b2) {
  const int lane = threadIdx.x & 31;
  const int c = L * LEAF + lane;
  const bool cv = c < P;
  const float cx = cv ? sx[c] : 0.0f, cy = cv ? sy[c] : 0.0f, cz = cv ? sz[c] : 0.0f;
  while (needmask) {
    const int q = __ffs(needmask) - 1;
    needmask &= needmask - 1;
    const float qx = __shfl_sync(0xffffffffu, px, q), qy = __shfl_sync(0xffffffffu, py, q);
    const float qz = __shfl_sync(0xffffffffu, pz, q), qb2 = __shfl_sync(0xffffffffu, b2, q);
    float d = FLT_BIG_K;
    if (cv) {
      const float dx = qx - cx, dy = qy - cy, dz = qz - cz;
      d = dx * dx + dy * dy + dz * dz;
    }
    float m[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      m[r] = warp_min(d);
      if (r == 0 && !(m[0] < qb2)) break;  // nothing below q's third-best: no change
      // drop one lane holding the minimum (a tie keeps its other copies)
      const unsigned at = __ballot_sync(0xffffffffu, d == m[r]);
      if (lane == __ffs(at) - 1) d = FLT_BIG_K;
      if (r == 0) {
        m[1] = m[2] = FLT_BIG_K;
      }
    }
    if (lane == q && m[0] < qb2) {
      push3(m[0], b0, b1, b2);
      push3(m[1], b0, b1, b2);
      push3(m[2], b0, b1, b2);
    }
  }
}

// Visits candidate leaf L (not the query's own) for the lanes whose lower
// bound to its box (cb, the same on every lane) does not exceed their third-best.
__device__ __forceinline__ void visit_leaf(int L, const float (&cb)[6], int P, bool valid, float px, float py,
                                           float pz, const float* __restrict__ sx, const float* __restrict__ sy,
                                           const float* __restrict__ sz, float4* s_pts, float& b0, float& b1,
                                           float& b2) {
  const bool need = valid && !(box_dist(cb, px, py, pz) > b2);
  const unsigned needmask = __ballot_sync(0xffffffffu, need);
  if (!needmask) return;
  if (__popc(needmask) <= SPARSE_LANES)
    scan_leaf_sparse(L, P, needmask, px, py, pz, sx, sy, sz, b0, b1, b2);
  else
    scan_leaf<false>(L, P, need, px, py, pz, sx, sy, sz, s_pts, b0, b1, b2);
}

// One warp per query leaf.  Boxes: leaves (nl), parents (np), grandparents (ng).
__global__ void __launch_bounds__(KT, 4) search_kernel(int P, int nl, int np, int ng, const float* __restrict__ sx,
                                                     const float* __restrict__ sy, const float* __restrict__ sz,
                                                     const float* __restrict__ leaf_b, const float* __restrict__ par_b,
                                                     const float* __restrict__ gp_b,
                                                     const unsigned* __restrict__ order, float* __restrict__ out) {
  __shared__ float4 s_leaf[KT / 32][32];
  const int lane = threadIdx.x & 31;
  const int qleaf = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  if (qleaf >= nl) return;  // whole warp
  float4* s_pts = s_leaf[threadIdx.x >> 5];
  const int my_idx = qleaf * LEAF + lane;
  const bool valid = my_idx < P;
  const float px = valid ? sx[my_idx] : 0.0f, py = valid ? sy[my_idx] : 0.0f, pz = valid ? sz[my_idx] : 0.0f;
  float b0 = FLT_BIG_K, b1 = FLT_BIG_K, b2 = FLT_BIG_K;
  // 1. the query's own leaf (its Morton neighbours): a first third-best.
  scan_leaf<true>(qleaf, P, valid, px, py, pz, sx, sy, sz, s_pts, b0, b1, b2);
  // 2. the two Morton-adjacent leaves: a query leaf that spans a jump of the
  // Morton curve holds the tail of one region and the head of another, whose
  // points continue in these two leaves, so every lane gets a close
  // third-best before the walks (which then skip both leaves).
#pragma unroll
  for (int side = -1; side <= 1; side += 2) {
    const int L = qleaf + side;
    if (L < 0 || L >= nl) continue;
    float cb[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) cb[k] = leaf_b[(size_t)L * 6 + k];
    visit_leaf(L, cb, P, valid, px, py, pz, sx, sy, sz, s_pts, b0, b1, b2);
  }
  float qb[6];  // the warp's query AABB
#pragma unroll
  for (int k = 0; k < 6; ++k) qb[k] = leaf_b[(size_t)qleaf * 6 + k];
  // 3. two walks over grandparents -> parents -> leaves, 32 boxes tested at a
  // time against the warp's query AABB: the first visits only leaves whose
  // box overlaps the query AABB (the local neighbourhood, which brings every
  // lane's third-best down quickly), the second every other leaf that its
  // lower bound does not rule out.  A leaf is scanned at most once: the
  // second walk skips exactly the leaves the first one visited.
  const int own_par = qleaf / 32, own_gp = own_par / 32;
  for (int pass = 0; pass < 2; ++pass) {
    // Grandparent g at box-box distance dgg from the query AABB: its parents,
    // then their leaves, that the pass's bound admits.
    auto visit_gp = [&](int g, float dgg) {
      float mb2 = pass == 0 ? 0.0f : warp_max(valid ? b2 : 0.0f);
      if (dgg > mb2) return;
      const int pidx = g * 32 + lane;
      float pbx[6];
#pragma unroll
      for (int k = 0; k < 6; ++k) pbx[k] = pidx < np ? par_b[(size_t)pidx * 6 + k] : 0.0f;
      unsigned pmask = __ballot_sync(0xffffffffu, pidx < np && boxbox_dist(qb, pbx) <= mb2);
      while (pmask) {
        const int pj = __ffs(pmask) - 1;
        const int pp = g * 32 + pj;
        pmask &= pmask - 1;
        // skip the parent when no lane's own bound reaches its box: no leaf
        // inside it can then be needed, now or later (third-bests only shrink)
        {
          float cb[6];
#pragma unroll
          for (int k = 0; k < 6; ++k) cb[k] = __shfl_sync(0xffffffffu, pbx[k], pj);
          if (!__any_sync(0xffffffffu, valid && !(box_dist(cb, px, py, pz) > b2))) continue;
        }
        if (pass == 1) mb2 = warp_max(valid ? b2 : 0.0f);
        // lane j holds leaf pp*32+j's box; the per-point test below takes it
        // by shuffle instead of a dependent load per visited leaf (a query
        // leaf spanning a Morton discontinuity overlaps thousands of leaves)
        const int lidx = pp * 32 + lane;
        float lb[6];
#pragma unroll
        for (int k = 0; k < 6; ++k) lb[k] = lidx < nl ? leaf_b[(size_t)lidx * 6 + k] : 0.0f;
        bool lneed = false;
        if (lidx < nl && (lidx < qleaf - 1 || lidx > qleaf + 1)) {
          const float d = boxbox_dist(qb, lb);
          lneed = pass == 0 ? d == 0.0f : (d > 0.0f && d <= mb2);
        }
        unsigned lmask = __ballot_sync(0xffffffffu, lneed);
        while (lmask) {
          const int j = __ffs(lmask) - 1;
          const int L = pp * 32 + j;
          lmask &= lmask - 1;
          float cb[6];
#pragma unroll
          for (int k = 0; k < 6; ++k) cb[k] = __shfl_sync(0xffffffffu, lb[k], j);
          visit_leaf(L, cb, P, valid, px, py, pz, sx, sy, sz, s_pts, b0, b1, b2);
        }
      }
    };
    // the query's own grandparent first, then the others in index order:
    // 32 grandparent distances per load (lane k holds grandparent 32c + k),
    // a ballot of those the bound admits at the chunk's start (a superset:
    // bounds only shrink, and visit_gp re-tests with the current one)
    {
      float tb[6];
#pragma unroll
      for (int k = 0; k < 6; ++k) tb[k] = gp_b[(size_t)own_gp * 6 + k];
      visit_gp(own_gp, boxbox_dist(qb, tb));
    }
    for (int c = 0; c * 32 < ng; ++c) {
      const int t = c * 32 + lane;
      float tb[6];
#pragma unroll
      for (int k = 0; k < 6; ++k) tb[k] = t < ng ? gp_b[(size_t)t * 6 + k] : 0.0f;
      const float dg = boxbox_dist(qb, tb);
      const float mb2c = pass == 0 ? 0.0f : warp_max(valid ? b2 : 0.0f);
      unsigned gmask = __ballot_sync(0xffffffffu, t < ng && t != own_gp && dg <= mb2c);
      while (gmask) {
        const int bit = __ffs(gmask) - 1;
        gmask &= gmask - 1;
        visit_gp(c * 32 + bit, __shfl_sync(0xffffffffu, dg, bit));
      }
    }
  }
  if (valid) out[order[my_idx]] = (b0 + b1 + b2) / 3.0f;
}

inline size_t a256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT size_t gsb_knn_workspace_bytes(int P) {
  const size_t n = (size_t)(P > 0 ? P : 1);
  const size_t nl = (n + LEAF - 1) / LEAF, np = (nl + 31) / 32, ng = (np + 31) / 32;
  size_t b = a256(n * 4) * 4;        // codes, codes_alt, idx, idx_alt
  b += a256(n * 4) * 3;              // sx, sy, sz
  b += a256(nl * 6 * 4) + a256(np * 6 * 4) + a256(ng * 6 * 4);  // leaf, parent, grandparent boxes
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
  const int nl = (P + LEAF - 1) / LEAF, np = (nl + 31) / 32, ng = (np + 31) / 32;
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
  float* leaf_b = (float*)take((size_t)nl * 6 * 4);
  float* par_b = (float*)take((size_t)np * 6 * 4);
  float* gp_b = (float*)take((size_t)ng * 6 * 4);
  float* part = (float*)take((size_t)BOUNDS_BLOCKS * 6 * 4);
  float* bounds = (float*)take(256);
  void* scratch = w;

  bounds_partial_kernel<<<BOUNDS_BLOCKS, KT, 0, s>>>(P, a->points, part);
  bounds_final_kernel<<<1, 32, 0, s>>>(BOUNDS_BLOCKS, part, bounds);
  morton_kernel<<<div_up(P, KT), KT, 0, s>>>(P, a->points, bounds, codes, idx);
  unsigned* kb[2] = {codes, codes_alt};
  unsigned* vb[2] = {idx, idx_alt};
  const int where = radix::sort_pairs(kb, vb, P, nullptr, 30, scratch, a->error_word, s);  // 30-bit Morton codes
  const unsigned* order = vb[where];
  gather_leaf_kernel<<<div_up((long long)nl * LEAF, KT), KT, 0, s>>>(P, a->points, order, sx, sy, sz, leaf_b);
  reduce_boxes_kernel<<<div_up((long long)np * 32, KT), KT, 0, s>>>(nl, leaf_b, par_b);
  reduce_boxes_kernel<<<div_up((long long)ng * 32, KT), KT, 0, s>>>(np, par_b, gp_b);
  search_kernel<<<div_up((long long)nl * 32, KT), KT, 0, s>>>(P, nl, np, ng, sx, sy, sz, leaf_b, par_b, gp_b,
                                                                order, a->out);
  return check_launch("gsb_knn");
}
