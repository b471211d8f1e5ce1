// binning.cu -- duplicate-with-keys, stable tile|depth ordering and tile ranges.
//
// Restates gswarp's _build_binning_state (binning_ops.py:84-431) in its
// default "warp_depth_stable_tile" form:
//   gsb_bin_count:     stable radix sort of all Gaussians by depth float bits
//                      (invisible ones last), gather of tiles_touched in that
//                      order and an inclusive scan (int64 total) -- the
//                      reference's K3/K7/K4/K5 (binning_ops.py:152-224).
//   gsb_bin_emit_sort: one thread per depth-ordered Gaussian re-runs the
//                      AccuTile sweep and writes (tile id, point id) pairs
//                      (binning_kernels.py:126-216, 410-451); a stable radix
//                      sort over ceil(log2(tiles)) key bits orders them by
//                      tile (memory.py:571-600); ranges come from the sorted
//                      keys (binning_kernels.py:467-487).
// The resulting point list is ordered by (tile, depth bits, point index), the
// canonical order both reference sort modes produce.  Built with -fmad=false
// so the emitted tiles match the preprocess counts bit for bit.
#include <algorithm>

#include "gsb_common.cuh"
#include "gsb_geometry.cuh"
#include "radix_sort.cuh"

namespace gsb {
namespace {

constexpr int SCAN_THREADS = launch::BINNING_SCAN;
constexpr int SCAN_ITEMS = 16;
constexpr int SCAN_TILE = SCAN_THREADS * SCAN_ITEMS;  // 4096

constexpr int SCAN_WARPS = SCAN_THREADS / 32;

// Decoupled look-back over one 62-bit value per tile, run by one warp: the
// warp reads 32 predecessors' status words at once, sums back to the nearest
// inclusive one and publishes this tile's inclusive value.  Tiles are claimed
// in launch order (atomic counter), so every tile waited on belongs to a
// running CTA; each spin is nevertheless bounded (SPIN_LIMIT): a timeout sets
// ERR_LOOKBACK_TIMEOUT and counts the slot as an inclusive zero, so the walk
// ends.  Returns the exclusive prefix (in every lane).
__device__ long long warp_lookback(unsigned long long* status, int tile, long long agg, long long* err) {
  using radix::FLAG_AGG;
  using radix::FLAG_INC;
  using radix::VALUE_MASK;
  const int lane = threadIdx.x & 31;
  if (lane == 0)
    radix::st_volatile(status + tile, (tile == 0 ? FLAG_INC : FLAG_AGG) | (unsigned long long)agg);
  long long excl = 0;
  if (tile > 0) {
    int t = tile - 1;
    while (true) {
      const int my = t - lane;
      unsigned long long v = FLAG_INC;  // before tile 0: an inclusive zero
      if (my >= 0) {
        v = radix::ld_volatile(status + my);
        int spins = 0;
        while ((v & ~VALUE_MASK) == 0 && ++spins < SPIN_LIMIT) v = radix::ld_volatile(status + my);
        if ((v & ~VALUE_MASK) == 0) {
          atomicOr((unsigned long long*)err, (unsigned long long)ERR_LOOKBACK_TIMEOUT);
          v = FLAG_INC;
        }
      }
      const unsigned inc = __ballot_sync(0xffffffffu, (v & ~VALUE_MASK) == FLAG_INC);
      const int stop = inc ? __ffs(inc) - 1 : 31;  // nearest inclusive predecessor
      long long val = lane <= stop ? (long long)(v & VALUE_MASK) : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) val += __shfl_xor_sync(0xffffffffu, val, o);
      excl += val;
      if (inc) break;
      t -= 32;
    }
    if (lane == 0) radix::st_volatile(status + tile, FLAG_INC | (unsigned long long)(excl + agg));
  }
  return excl;
}

// Order-preserving compaction of the Gaussians with tiles in one pass:
// keys = depth float bits, vals = point index, in index order (so the stable
// depth sort breaks depth ties by index).  A CTA takes 4096 consecutive
// Gaussians as 16 chunks of 256; positions inside the CTA come from per-warp
// ballots, the CTA's offset from the look-back.  The last tile writes the
// count V.
__global__ void __launch_bounds__(SCAN_THREADS) compact_kernel(
    int P, const float* __restrict__ depths, const int* __restrict__ tiles_touched,
    unsigned long long* __restrict__ status, unsigned* __restrict__ counter, unsigned* __restrict__ keys,
    unsigned* __restrict__ vals, int* __restrict__ ids_out, long long* __restrict__ count_out,
    int* __restrict__ count_int, long long* __restrict__ err) {
  __shared__ int s_tile;
  __shared__ int s_pre[SCAN_ITEMS * SCAN_WARPS];
  __shared__ int s_wsum[SCAN_WARPS];
  __shared__ long long s_excl;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_tile = (int)atomicAdd(counter, 1u);
  __syncthreads();
  const int tile = s_tile;
  const long long base = (long long)tile * SCAN_TILE;
  unsigned m[SCAN_ITEMS];
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    const long long r = base + i * SCAN_THREADS + tid;
    m[i] = __ballot_sync(0xffffffffu, r < P && tiles_touched[r] > 0);
    if (lane == 0) s_pre[i * SCAN_WARPS + warp] = __popc(m[i]);
  }
  __syncthreads();
  // exclusive prefix over the (chunk, warp) counts in index order
  const int v = tid < SCAN_ITEMS * SCAN_WARPS ? s_pre[tid] : 0;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_wsum[warp] = x;
  __syncthreads();
  int wpre = 0, total = 0;
#pragma unroll
  for (int w = 0; w < SCAN_WARPS; ++w) {
    wpre += w < warp ? s_wsum[w] : 0;
    total += s_wsum[w];
  }
  if (tid < SCAN_ITEMS * SCAN_WARPS) s_pre[tid] = wpre + x - v;
  if (warp == 0) {
    const long long e = warp_lookback(status, tile, total, err);
    if (lane == 0) s_excl = e;
  }
  __syncthreads();
  const long long excl = s_excl;
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    if ((m[i] >> lane) & 1u) {
      const long long r = base + i * SCAN_THREADS + tid;
      const long long o = excl + s_pre[i * SCAN_WARPS + warp] + __popc(m[i] & lt);
      keys[o] = __float_as_uint(depths[r]);
      vals[o] = (unsigned)r;
      if (ids_out) ids_out[o] = (int)r;
    }
  }
  if (tile == (int)gridDim.x - 1 && tid == 0) {
    count_out[0] = excl + total;
    *count_int = (int)(excl + total);
  }
}

// Inclusive scan of tiles_touched in depth order in one pass:
// offsets[r] = sum_{q<=r} tiles[order[q]] over the first n = *n_dev entries.
// Ids are read coalesced, the counts gathered, and each thread scans 16
// consecutive counts through shared memory (padded: conflict-free); the
// CTA's offset comes from the look-back; the tile holding the last entry
// writes the int64 total.
__global__ void __launch_bounds__(SCAN_THREADS) depth_scan_kernel(
    const int* __restrict__ n_dev, const int* __restrict__ order, const int* __restrict__ tiles_touched,
    unsigned long long* __restrict__ status, unsigned* __restrict__ counter, int* __restrict__ offsets,
    long long* __restrict__ total_out, long long* __restrict__ err) {
  constexpr int PAD = SCAN_TILE + SCAN_TILE / 16;
  __shared__ int s_c[PAD];
  __shared__ long long s_wsum[SCAN_WARPS];
  __shared__ long long s_excl;
  __shared__ int s_tile;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = *n_dev;
  if (tid == 0) s_tile = (int)atomicAdd(counter, 1u);
  __syncthreads();
  const int tile = s_tile;
  const long long base = (long long)tile * SCAN_TILE;
  if (base >= n) return;  // every later tile lies past n as well: nobody waits on this one
  int c[SCAN_ITEMS];
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    const long long r = base + i * SCAN_THREADS + tid;
    c[i] = r < n ? order[r] : -1;
  }
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) c[i] = c[i] >= 0 ? tiles_touched[c[i]] : 0;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    const int l = i * SCAN_THREADS + tid;
    s_c[l + l / 16] = c[i];
  }
  __syncthreads();
  long long run = 0;
  long long mine[SCAN_ITEMS];
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    run += s_c[tid * 17 + i];  // local index tid*16 + i, padded
    mine[i] = run;
  }
  long long x = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_wsum[warp] = x;
  __syncthreads();
  long long wpre = 0, total = 0;
#pragma unroll
  for (int w = 0; w < SCAN_WARPS; ++w) {
    wpre += w < warp ? s_wsum[w] : 0;
    total += s_wsum[w];
  }
  if (warp == 0) {
    const long long e = warp_lookback(status, tile, total, err);
    if (lane == 0) s_excl = e;
  }
  __syncthreads();
  const long long pre = s_excl + wpre + x - run;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) s_c[tid * 17 + i] = (int)(pre + mine[i]);
  __syncthreads();
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; ++i) {
    const int l = i * SCAN_THREADS + tid;
    const long long r = base + l;
    if (r < n) offsets[r] = s_c[l + l / 16];
  }
  if (base + SCAN_TILE >= n && tid == 0) *total_out = s_excl + total;
}

struct EmitPairs {
  unsigned* keys;
  unsigned* vals;
  long long start;
  int cap;
  int point;
  mutable int k;
  __device__ __forceinline__ void operator()(int tile) const {
    if (k < cap) {
      keys[start + k] = (unsigned)tile;
      vals[start + k] = (unsigned)point;
    }
    ++k;
  }
};

// Emit from the 32-byte binning records written by preprocess, one warp per
// 32 consecutive depth-ordered Gaussians.  Each lane reads its Gaussian's
// record (one random 32-byte read) and pair count (the difference of
// adjacent inclusive offsets), the warp scans the counts, and then the lanes
// take consecutive pairs of the warp -- the owning Gaussian found by binary
// search over the warp's prefix, the tile decoded from its record -- so every
// store is coalesced and no lane waits for the warp's largest footprint.
// Records with more than BINREC_MAX_BANDS bands re-run the sweep from the
// render record per lane afterwards.  A record whose tile count differs from
// the pair count raises ERR_EMIT_MISMATCH (and emits no more than the count).
// Slots of the pair count that a mismatching record does not fill get the
// key EMIT_FILL_KEY (no tile: above every tile id, so the ranges pass skips
// it) and the Gaussian's own id, so nothing downstream reads an
// uninitialised key or point id.
constexpr unsigned EMIT_FILL_KEY = 0xFFFFFFFFu;

__device__ __forceinline__ void emit_fill(unsigned* keys, unsigned* vals, long long start, int from, int n,
                                          int point) {
  for (int k = from; k < n; ++k) {
    keys[start + k] = EMIT_FILL_KEY;
    vals[start + k] = (unsigned)point;
  }
}

struct EmitLane {
  unsigned w[8];
  int pre, start, point;
};

__device__ __forceinline__ int record_count(const unsigned (&w)[8]) {
  const int x0 = (int)(w[0] & 0xFFFFu), y0 = (int)(w[0] >> 16);
  const int x1 = (int)(w[1] & 0xFFFFu), y1 = (int)(w[1] >> 16);
  const unsigned kind = w[2] & 3u;
  if (kind == BINREC_RECT) return (x1 - x0) * (y1 - y0);
  if (kind == BINREC_MASK) return __popc(w[3]) + __popc(w[4]);
  int c = 0;
  const int nb = (int)((w[2] >> 8) & 0xFFu);
  for (int b = 0; b < nb && b < BINREC_MAX_BANDS; ++b) c += imx(0, (int)(w[3 + b] >> 16) - (int)(w[3 + b] & 0xFFFFu));
  return c;
}

// Tile of the idx-th pair of a (non-sweep) record, in cover_tiles_in_rect's order.
__device__ __forceinline__ int record_tile(const unsigned* w, int idx, int gx) {
  const int x0 = (int)(w[0] & 0xFFFFu), y0 = (int)(w[0] >> 16);
  const int x1 = (int)(w[1] & 0xFFFFu);
  const unsigned kind = w[2] & 3u;
  const int width = x1 - x0;
  if (kind == BINREC_RECT) {
    const int row = idx / width;
    return (y0 + row) * gx + x0 + (idx - row * width);
  }
  if (kind == BINREC_MASK) {
    const int lo = __popc(w[3]);
    const int bit = idx < lo ? __fns(w[3], 0, idx + 1) : 32 + __fns(w[4], 0, idx - lo + 1);
    const int row = bit / width;
    return (y0 + row) * gx + x0 + (bit - row * width);
  }
  const bool vertical = (w[2] >> 2) & 1u;
  const int nb = (int)((w[2] >> 8) & 0xFFu);
  for (int b = 0; b < nb; ++b) {
    const int lo = (int)(w[3 + b] & 0xFFFFu), hi = (int)(w[3 + b] >> 16);
    const int len = imx(0, hi - lo);
    if (idx < len) return vertical ? (lo + idx) * gx + x0 + b : (y0 + b) * gx + lo + idx;
    idx -= len;
  }
  return 0;  // unreachable: idx < record_count
}

constexpr int EMIT_THREADS = launch::BINNING_EMIT;

__global__ void __launch_bounds__(EMIT_THREADS, 8) emit_binrec_kernel(
    const long long* __restrict__ n_dev, int gx, int mode, const int* __restrict__ order,
    const int* __restrict__ offsets, const uint4* __restrict__ bin_records, const float4* __restrict__ records,
    unsigned* __restrict__ keys, unsigned* __restrict__ vals, long long* __restrict__ err) {
  __shared__ EmitLane s_lane[EMIT_THREADS];
  const int lane = threadIdx.x & 31;
  const long long nv = *n_dev;
  const long long warp_first = ((long long)blockIdx.x * EMIT_THREADS + (threadIdx.x & ~31));
  if (warp_first >= nv) return;  // whole warp past the binned Gaussians
  const int r = (int)(warp_first + lane);
  EmitLane& me = s_lane[threadIdx.x];
  int n = 0, point = 0, start = 0;
  unsigned w[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
  if (r < nv) {
    // the id is read with the offsets (not after them): one round trip less
    // before the record load
    point = order[r];
    const int end = offsets[r];
    n = end - (r > 0 ? offsets[r - 1] : 0);
    start = end - n;
    if (n > 0) {
      const uint4 a = __ldg(bin_records + (size_t)point * 2), b = __ldg(bin_records + (size_t)point * 2 + 1);
      w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
      w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
  }
  const bool sweep = n > 0 && (w[2] & 3u) == BINREC_SWEEP;
  int ncoop = 0;
  if (n > 0 && !sweep) {
    const int c = record_count(w);
    if (c != n) atomicOr((unsigned long long*)err, (unsigned long long)ERR_EMIT_MISMATCH);
    ncoop = min(c, n);
  }
  // warp exclusive scan of the cooperative counts
  int x = ncoop;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  const int total = __shfl_sync(0xffffffffu, x, 31);
#pragma unroll
  for (int k = 0; k < 8; ++k) me.w[k] = w[k];
  me.pre = x - ncoop;
  me.start = start;
  me.point = point;
  __syncwarp();
  const EmitLane* wl = s_lane + (threadIdx.x & ~31);
  for (int q = lane; q < total; q += 32) {
    // owner: the last lane whose prefix is <= q (a lane after the owner starts past q; lanes
    // without pairs before it have lower indices)
    int o = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1)
      if (wl[o + step].pre <= q) o += step;
    const int idx = q - wl[o].pre;
    const int pos = wl[o].start + idx;
    keys[pos] = (unsigned)record_tile(wl[o].w, idx, gx);
    vals[pos] = (unsigned)wl[o].point;
  }
  if (n > 0 && !sweep && ncoop < n) emit_fill(keys, vals, start, ncoop, n, point);
  if (sweep) {
    const float4 q0 = __ldg(records + (size_t)point * 3), q1 = __ldg(records + (size_t)point * 3 + 1);
    const float t = opacity_threshold(q1.y);
    EmitPairs e{keys, vals, (long long)start, n, point, 0};
    emit_record(w, gx, mode, q0.x, q0.y, q0.z, q0.w, q1.x, t, e);
    if (e.k != n) atomicOr((unsigned long long*)err, (unsigned long long)ERR_EMIT_MISMATCH);
    if (e.k < n) emit_fill(keys, vals, start, e.k, n, point);
  }
}

__global__ void __launch_bounds__(256) emit_kernel(
    const long long* __restrict__ n_dev, int gx, int gy, int mode, const int* __restrict__ order,
    const int* __restrict__ offsets, const int* __restrict__ tiles_touched,
    const int* __restrict__ radii, const float4* __restrict__ records,
    const float* __restrict__ conic_2d_inv, unsigned* __restrict__ keys,
    unsigned* __restrict__ vals, long long* __restrict__ err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= *n_dev) return;
  const int p = order[r];
  // the slots are the ones the offsets give this Gaussian (as in the record
  // path); a coverage that produces another count is flagged and filled
  const int end = offsets[r];
  const int n = end - (r > 0 ? offsets[r - 1] : 0);
  if (n <= 0) return;
  const int radius = radii[p];
  const float4 q0 = records[(size_t)p * 3 + 0];
  const float4 q1 = records[(size_t)p * 3 + 1];
  const float cov_a = conic_2d_inv[(size_t)p * 3 + 0];
  const float cov_c = conic_2d_inv[(size_t)p * 3 + 2];
  EmitPairs e{keys, vals, (long long)end - n, n, p, 0};
  cover_tiles(q0.x, q0.y, cov_a, cov_c, q0.z, q0.w, q1.x, q1.y, radius, gx, gy, mode, e);
  if (e.k != n) atomicOr((unsigned long long*)err, (unsigned long long)ERR_EMIT_MISMATCH);
  if (e.k < n) emit_fill(keys, vals, e.start, e.k, n, p);
}


inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// Ranges when the sort has no pass to write them: a single tile (every key
// is 0) or a single pair.
__global__ void single_range_kernel(const unsigned* __restrict__ keys, int R, int tiles, int* __restrict__ ranges) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const unsigned k = keys[0];
    if (k >= (unsigned)tiles) return;  // an emit fill key (mismatch flagged): no range
    ranges[2 * (size_t)k] = 0;
    ranges[2 * (size_t)k + 1] = R;
  }
}

// Significant bits of a tile id (0 for a single tile) and the sort passes they take.
inline int tile_key_bits(int tiles) { return tiles <= 1 ? 0 : 32 - __builtin_clz((unsigned)(tiles - 1)); }
inline int tile_sort_passes(int tiles) { return radix::passes_for_bits(tile_key_bits(tiles)); }

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT size_t gsb_bin_count_workspace_bytes(int P) {
  const size_t n = (size_t)(P > 0 ? P : 1);
  size_t b = 0;
  b += align256(n * 4) * 3;  // keys, keys_alt, vals_alt
  b += align256((size_t)div_up((long long)n, SCAN_TILE) * 8) * 2;  // look-back status of the two scans
  b += 256;                  // device count of Gaussians with tiles, tile counters
  b += radix::scratch_bytes((long long)n, 4);
  return b + 256;
}

GSB_EXPORT int gsb_bin_count(const gsb_bin_count_args* a, void* stream) {
  if (!a || a->P < 0) {
    set_error("gsb_bin_count: invalid arguments");
    return GSB_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (!a->status_out) {
    set_error("gsb_bin_count: status_out is required");
    return GSB_ERR_INVALID;
  }
  if (a->P == 0) {
    cudaMemsetAsync(a->status_out, 0, 3 * sizeof(long long), s);
    return check_launch("gsb_bin_count(empty)");
  }
  if (!a->depths || !a->radii || !a->tiles_touched || !a->depth_order || !a->point_offsets ||
      !a->workspace || a->workspace_bytes < gsb_bin_count_workspace_bytes(a->P)) {
    set_error("gsb_bin_count: null pointer or workspace too small");
    return GSB_ERR_INVALID;
  }
  const int P = a->P;
  char* w = (char*)(((uintptr_t)a->workspace + 255) & ~(uintptr_t)255);
  unsigned* keys = (unsigned*)w;
  w += align256((size_t)P * 4);
  unsigned* keys_alt = (unsigned*)w;
  w += align256((size_t)P * 4);
  unsigned* vals_alt = (unsigned*)w;
  w += align256((size_t)P * 4);
  const int nblocks = div_up(P, SCAN_TILE);
  const size_t status_bytes = align256((size_t)nblocks * 8);
  unsigned long long* status_c = (unsigned long long*)w;
  unsigned long long* status_s = (unsigned long long*)(w + status_bytes);
  w += 2 * status_bytes;
  int* n_vis = (int*)w;
  unsigned* counters = (unsigned*)(w + 16);  // [0] compaction, [1] scan
  w += 256;
  void* sort_scratch = w;

  long long* err = a->status_out + 1;
  // look-back status words and tile counters start at zero; so do the pair
  // total and the error word (V is always written)
  cudaMemsetAsync(status_c, 0, 2 * status_bytes + 256, s);
  cudaMemsetAsync(a->status_out, 0, 2 * sizeof(long long), s);
  // 1. order-preserving compaction of the Gaussians with tiles (count V into
  //    status_out[2] and n_vis); only they take part in the depth sort.
  unsigned* vals0 = (unsigned*)a->depth_order;
  compact_kernel<<<nblocks, SCAN_THREADS, 0, s>>>(P, a->depths, a->tiles_touched, status_c, counters, keys, vals0,
                                                  a->binned_ids, a->status_out + 2, n_vis, err);
  // 2. stable sort of the V (depth bits, index) pairs.
  unsigned* kb[2] = {keys, keys_alt};
  unsigned* vb[2] = {vals0, vals_alt};
  const int where = radix::sort_pairs(kb, vb, P, n_vis, 32, sort_scratch, err, s);
  if (where != 0) {  // 4 passes always end in buffer 0; kept for safety
    cudaMemcpyAsync(a->depth_order, vals_alt, (size_t)P * 4, cudaMemcpyDeviceToDevice, s);
  }
  // 3. inclusive scan of tiles_touched in depth order; pair total -> status_out[0].
  depth_scan_kernel<<<nblocks, SCAN_THREADS, 0, s>>>(n_vis, a->depth_order, a->tiles_touched, status_s, counters + 1,
                                                     a->point_offsets, a->status_out, err);
  return check_launch("gsb_bin_count");
}

GSB_EXPORT size_t gsb_bin_sort_workspace_bytes(long long R, int W, int H) {
  const int tiles = div_up(W, BLOCK_X) * div_up(H, BLOCK_Y);
  const size_t n = (size_t)(R > 0 ? R : 1);
  size_t b = align256(n * 4) * 3;  // keys, keys_alt, vals_alt
  b += radix::scratch_bytes((long long)n, std::max(tile_sort_passes(tiles), 1));
  return b + 256;
}

GSB_EXPORT int gsb_bin_emit_sort(const gsb_bin_sort_args* a, void* stream) {
  if (!a || a->P < 0 || a->W <= 0 || a->H <= 0 || a->num_rendered < 0 ||
      a->num_rendered > 2147483647ll) {
    set_error("gsb_bin_emit_sort: invalid sizes");
    return a && a->num_rendered > 2147483647ll ? GSB_ERR_OVERFLOW : GSB_ERR_INVALID;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const int gx = div_up(a->W, BLOCK_X), gy = div_up(a->H, BLOCK_Y);
  const int tiles = gx * gy;
  if (!a->ranges || !a->error_word || !a->bin_status) {
    set_error("gsb_bin_emit_sort: ranges, error_word and bin_status are required");
    return GSB_ERR_INVALID;
  }
  cudaMemsetAsync(a->ranges, 0, (size_t)tiles * 2 * sizeof(int), s);
  const long long R = a->num_rendered;
  if (R == 0 || a->P == 0) return check_launch("gsb_bin_emit_sort(empty)");
  const bool binrec = a->bin_records != nullptr;
  if (!a->depth_order || !a->point_offsets || !a->point_list || !a->workspace ||
      !a->records || (!binrec && (!a->radii || !a->conic_2d_inv || !a->tiles_touched)) ||
      a->workspace_bytes < gsb_bin_sort_workspace_bytes(R, a->W, a->H)) {
    set_error("gsb_bin_emit_sort: null pointer or workspace too small");
    return GSB_ERR_INVALID;
  }
  if (binrec && ((reinterpret_cast<uintptr_t>(a->bin_records) & 15) || gx > 65535 || gy > 65535)) {
    set_error("gsb_bin_emit_sort: bin_records needs 16-byte alignment and tile grids below 65536");
    return GSB_ERR_INVALID;
  }
  char* w = (char*)(((uintptr_t)a->workspace + 255) & ~(uintptr_t)255);
  unsigned* keys = (unsigned*)w;
  w += align256((size_t)R * 4);
  unsigned* keys_alt = (unsigned*)w;
  w += align256((size_t)R * 4);
  unsigned* vals_alt = (unsigned*)w;
  w += align256((size_t)R * 4);
  void* sort_scratch = w;

  const int passes = tile_sort_passes(tiles);
  // Emit into whichever value buffer the last sort pass will NOT write, so
  // the sorted point ids land directly in point_list.
  unsigned* pl = (unsigned*)a->point_list;
  unsigned* vb[2];
  unsigned* kb[2] = {keys, keys_alt};
  if (passes % 2 == 0) {
    vb[0] = pl;
    vb[1] = vals_alt;
  } else {
    vb[0] = vals_alt;
    vb[1] = pl;
  }
  if (binrec)
    emit_binrec_kernel<<<div_up(a->P, EMIT_THREADS), EMIT_THREADS, 0, s>>>(
        a->bin_status + 2, gx, a->coverage_mode, a->depth_order, a->point_offsets,
        reinterpret_cast<const uint4*>(a->bin_records), reinterpret_cast<const float4*>(a->records), kb[0],
        vb[0], a->error_word);
  else
    emit_kernel<<<div_up(a->P, 256), 256, 0, s>>>(
        a->bin_status + 2, gx, gy, a->coverage_mode, a->depth_order, a->point_offsets, a->tiles_touched, a->radii,
        reinterpret_cast<const float4*>(a->records), a->conic_2d_inv, kb[0], vb[0], a->error_word);
  // the last pass also writes the per-tile ranges (the array was zeroed above)
  if (passes == 0 || R <= 1) {
    // nothing to sort: the emitted order is the sorted order
    if (vb[0] != pl) cudaMemcpyAsync(pl, vb[0], (size_t)R * 4, cudaMemcpyDeviceToDevice, s);
    single_range_kernel<<<1, 32, 0, s>>>(kb[0], (int)R, tiles, a->ranges);
  } else
    radix::sort_pairs(kb, vb, R, nullptr, tile_key_bits(tiles), sort_scratch, a->error_word, s, a->ranges, tiles);
  return check_launch("gsb_bin_emit_sort");
}
