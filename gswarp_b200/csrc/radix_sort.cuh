// radix_sort.cuh -- stable LSD radix sort of (uint32 key, uint32 value) pairs.
//
// Replaces Warp's wp.utils.radix_sort_pairs (called from gswarp
// memory.py:571-600 and knn.py:337-341) with a reduce-then-scan design for
// sm_100a, 8 key bits a pass:
//   1. one histogram kernel computes the digit histograms of every pass in a
//      single read of the keys (per-warp shared sub-histograms);
//   2. a tiny kernel turns them into per-pass bin bases;
//   3. each pass: a count kernel writes every 3840-key tile's digit counts,
//      a scan kernel (a CTA per digit) turns them into the tiles' output
//      offsets, and a scatter kernel ranks each tile's keys stably per warp
//      (per-bit ballots), stages the tile in digit order in shared memory
//      and writes it out in runs.
// No CTA waits on another (the offsets are known before the scatter starts),
// at the cost of reading the keys once more per pass.
#pragma once

#include <algorithm>

#include "gsb_common.cuh"

namespace gsb {
namespace radix {
// Internal linkage: every translation unit that sorts gets its own copy.
namespace {

constexpr int RADIX_BITS = 8;
constexpr int RADIX = 1 << RADIX_BITS;
constexpr int THREADS = launch::RADIX_SORT;
constexpr int WARPS = THREADS / 32;
constexpr int ITEMS = 15;
constexpr int TILE_KEYS = THREADS * ITEMS;  // 3840
constexpr int MAX_PASSES = 4;
constexpr int HIST_ITEMS = 8;

constexpr unsigned long long FLAG_AGG = 1ull << 62;
constexpr unsigned long long FLAG_INC = 2ull << 62;
constexpr unsigned long long VALUE_MASK = (1ull << 62) - 1;

__device__ __forceinline__ unsigned long long ld_volatile(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Lanes of the warp whose 9-bit value d (an 8-bit digit, or RADIX for "no
// key") equals this lane's: nine ballots, one per bit (cheaper on sm_100a
// than a match.any over 32 distinct values).
__device__ __forceinline__ unsigned digit_peers(unsigned d) {
  unsigned peers = 0xffffffffu;
#pragma unroll
  for (int b = 0; b <= RADIX_BITS; ++b) {
    const bool bit = (d >> b) & 1u;
    const unsigned m = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? m : ~m;
  }
  return peers;
}

// Exclusive scan of one value per thread across a 256-thread CTA.
__device__ __forceinline__ unsigned block_exclusive_scan(unsigned v, unsigned* s_warp,
                                                         unsigned* total_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  unsigned wpre = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) {
    unsigned t = s_warp[w];
    if (w < warp) wpre += t;
    tot += t;
  }
  __syncthreads();
  if (total_out) *total_out = tot;
  return wpre + x - v;
}

// Digit histograms of every pass in one read of the keys.  Each warp counts
// into its own shared sub-histogram with plain shared atomics (same-digit
// lanes serialize in hardware; digits of depth bits and tile ids spread well
// enough that this beats aggregating peers first), HIST_ITEMS keys per lane
// loaded before any is counted.
__global__ void __launch_bounds__(THREADS) histogram_kernel(const unsigned* __restrict__ keys,
                                                            int n_host, const int* __restrict__ n_dev,
                                                            int passes, unsigned* __restrict__ hist) {
  const int n = n_dev ? *n_dev : n_host;
  __shared__ unsigned s_hist[WARPS][MAX_PASSES][RADIX];
  for (int i = threadIdx.x; i < WARPS * MAX_PASSES * RADIX; i += THREADS) (&s_hist[0][0][0])[i] = 0u;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long warps_total = (long long)gridDim.x * WARPS;
  const long long warp_id = (long long)blockIdx.x * WARPS + warp;
  for (long long base = warp_id * 32 * HIST_ITEMS; base < n; base += warps_total * 32 * HIST_ITEMS) {
    unsigned kv[HIST_ITEMS];
#pragma unroll
    for (int it = 0; it < HIST_ITEMS; ++it) {
      const long long i = base + it * 32 + lane;
      kv[it] = i < n ? __ldg(keys + i) : 0u;
    }
#pragma unroll
    for (int it = 0; it < HIST_ITEMS; ++it) {
      if (base + it * 32 + lane < n) {
        for (int p = 0; p < passes; ++p)
          atomicAdd(&s_hist[warp][p][(kv[it] >> (p * RADIX_BITS)) & (RADIX - 1)], 1u);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * RADIX; i += THREADS) {
    unsigned c = 0;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) c += (&s_hist[w][0][0])[i];
    if (c) atomicAdd(&hist[i], c);
  }
}

__global__ void __launch_bounds__(THREADS) bin_base_kernel(const unsigned* __restrict__ hist,
                                                           unsigned* __restrict__ bin_base) {
  __shared__ unsigned s_warp[WARPS];
  const int p = blockIdx.x;
  const unsigned c = hist[p * RADIX + threadIdx.x];
  bin_base[p * RADIX + threadIdx.x] = block_exclusive_scan(c, s_warp, nullptr);
}

// Pass step 1: every tile's digit counts, digit-major (counts[d * tiles + t]),
// zero for tiles past the element count.
__global__ void __launch_bounds__(THREADS) tile_count_kernel(const unsigned* __restrict__ keys, int n_host,
                                                             const int* __restrict__ n_dev, int shift,
                                                             unsigned* __restrict__ counts, int tiles) {
  __shared__ unsigned s_count[RADIX];
  const int tid = threadIdx.x;
  const int n = n_dev ? *n_dev : n_host;
  s_count[tid] = 0u;
  __syncthreads();
  const long long base = (long long)blockIdx.x * TILE_KEYS;
  unsigned key[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const long long pos = base + i * THREADS + tid;
    key[i] = pos < n ? __ldg(keys + pos) : 0u;
  }
#pragma unroll
  for (int i = 0; i < ITEMS; ++i)
    if (base + i * THREADS + tid < n) atomicAdd(&s_count[(key[i] >> shift) & (RADIX - 1)], 1u);
  __syncthreads();
  counts[(size_t)tid * tiles + blockIdx.x] = s_count[tid];
}

// Pass step 2: one CTA per digit turns its row of tile counts into the
// tiles' global output offsets for that digit: the digit's base (all keys of
// smaller digits) plus an exclusive scan over the tiles, in place.
__global__ void __launch_bounds__(THREADS) tile_offset_kernel(unsigned* __restrict__ counts, int tiles,
                                                              const unsigned* __restrict__ bin_base) {
  __shared__ unsigned s_warp[WARPS];
  unsigned* row = counts + (size_t)blockIdx.x * tiles;
  unsigned carry = bin_base[blockIdx.x];
  for (int t0 = 0; t0 < tiles; t0 += THREADS) {
    const int t = t0 + threadIdx.x;
    const unsigned c = t < tiles ? row[t] : 0u;
    unsigned total;
    const unsigned ex = block_exclusive_scan(c, s_warp, &total);
    if (t < tiles) row[t] = carry + ex;
    carry += total;
  }
}

// Pass step 3: a CTA per tile ranks its keys stably per warp (per-bit
// ballots, the rounds of a warp holding consecutive keys), stages the tile in
// digit order in shared memory and writes it out in runs at the offsets of
// step 2.  No tile waits on another.
template <bool HAS_VALS>
__global__ void __launch_bounds__(THREADS, 4) scatter_kernel(
    const unsigned* __restrict__ keys_in, const unsigned* __restrict__ vals_in,
    unsigned* __restrict__ keys_out, unsigned* __restrict__ vals_out, int n_host,
    const int* __restrict__ n_dev, int shift, const unsigned* __restrict__ offsets, int tiles,
    int* __restrict__ ranges, int range_keys) {
  __shared__ unsigned s_keys[TILE_KEYS];
  __shared__ unsigned s_vals[HAS_VALS ? TILE_KEYS : 1];
  __shared__ unsigned s_warp_hist[WARPS][RADIX];
  __shared__ unsigned s_digit_start[RADIX];
  __shared__ unsigned s_global[RADIX];
  __shared__ unsigned s_scan[WARPS];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // With a device-side count the grid is sized for the upper bound.
  const int n = n_dev ? *n_dev : n_host;
  const int tile = blockIdx.x;
  if ((long long)tile * TILE_KEYS >= n) return;
  for (int i = tid; i < WARPS * RADIX; i += THREADS) (&s_warp_hist[0][0])[i] = 0u;
  s_global[tid] = offsets[(size_t)tid * tiles + tile];
  __syncthreads();
  const long long base = (long long)tile * TILE_KEYS + (long long)warp * (ITEMS * 32);

  unsigned key[ITEMS], rank[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const long long pos = base + i * 32 + lane;
    const bool valid = pos < n;
    key[i] = valid ? keys_in[pos] : 0xFFFFFFFFu;
    rank[i] = valid ? 0u : 0xFFFFFFFFu;  // invalid marker
  }
  // Stable warp-local ranking: round i holds 32 consecutive keys.  The
  // lowest lane of each digit group adds the group's size to the warp's
  // counter with a shared atomic and hands the old count to its peers: no
  // read-then-write chain between rounds (shared atomics of one warp to one
  // address take effect in issue order, so rounds keep their order).
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const bool valid = rank[i] != 0xFFFFFFFFu;
    const unsigned d = valid ? (key[i] >> shift) & (RADIX - 1) : (unsigned)RADIX;
    const unsigned peers = digit_peers(d);
    const int leader = __ffs(peers) - 1;
    unsigned old = 0;
    if (valid && lane == leader) old = atomicAdd(&s_warp_hist[warp][d], (unsigned)__popc(peers));
    old = __shfl_sync(0xffffffffu, old, leader);
    if (valid) rank[i] = old + __popc(peers & lt);
  }
  __syncthreads();

  // Thread `tid` owns digit `tid`: per-warp exclusive offsets and tile count.
  unsigned total = 0;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) {
    const unsigned c = s_warp_hist[w][tid];
    s_warp_hist[w][tid] = total;
    total += c;
  }
  s_digit_start[tid] = block_exclusive_scan(total, s_scan, nullptr);
  __syncthreads();

  // Stage the tile in digit order; values are read here, not earlier.
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    if (rank[i] != 0xFFFFFFFFu) {
      const unsigned d = (key[i] >> shift) & (RADIX - 1);
      rank[i] += s_digit_start[d] + s_warp_hist[warp][d];
      s_keys[rank[i]] = key[i];
    }
  }
  if (HAS_VALS) {
    unsigned val[ITEMS];
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const long long pos = base + i * 32 + lane;
      val[i] = rank[i] != 0xFFFFFFFFu ? vals_in[pos] : 0u;
    }
#pragma unroll
    for (int i = 0; i < ITEMS; ++i)
      if (rank[i] != 0xFFFFFFFFu) s_vals[rank[i]] = val[i];
  }
  __syncthreads();
  const long long tile_base = (long long)tile * TILE_KEYS;
  const int tile_n = (int)min((long long)TILE_KEYS, (long long)n - tile_base);
  for (int j = tid; j < tile_n; j += THREADS) {
    const unsigned k = s_keys[j];
    const unsigned d = (k >> shift) & (RADIX - 1);
    const unsigned dst = s_global[d] + (unsigned)j - s_digit_start[d];
    // dst < n whenever the counts and the keys agree (the test keeps any
    // write inside the output)
    if (dst < (unsigned)n) {
      keys_out[dst] = k;
      if (HAS_VALS) vals_out[dst] = s_vals[j];
      if (ranges) {
        // Last pass: the staged tile is sorted by the whole key, so a key
        // whose neighbour in the tile differs is the tile's first / last
        // occurrence of it.  The key's global [start, end) is the min / max
        // over the tiles that hold it: end by atomicMax, start as n - start
        // by atomicMax (both fields start at zero, so keys that never occur
        // stay (0, 0)); ranges_fixup_kernel turns n - start back into start.
        // Keys at or above range_keys (the emit's fill for pairs it could not
        // produce, flagged in the error word) have no range slot.
        if (k < (unsigned)range_keys) {
          if (j == 0 || s_keys[j - 1] != k) atomicMax(ranges + 2 * (size_t)k, n - (int)dst);
          if (j == tile_n - 1 || s_keys[j + 1] != k) atomicMax(ranges + 2 * (size_t)k + 1, (int)dst + 1);
        }
      }
    }
  }
}

__global__ void ranges_fixup_kernel(int keys, int n, int* __restrict__ ranges) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < keys && ranges[2 * k + 1] > 0) ranges[2 * k] = n - ranges[2 * k];
}

// Workspace layout for sorting n pairs with `passes` 8-bit passes.
struct SortScratch {
  unsigned* hist;      // passes*256
  unsigned* bin_base;  // passes*256
  unsigned* counts;    // 256*tiles, reused by every pass
  size_t zero_bytes;   // bytes to clear from `hist` on
};

__host__ inline int num_tiles(long long n) { return (int)((n + TILE_KEYS - 1) / TILE_KEYS); }

__host__ inline size_t scratch_bytes(long long n, int passes) {
  const size_t tiles = (size_t)num_tiles(n > 0 ? n : 1);
  size_t b = 0;
  b += (size_t)passes * RADIX * 4;  // hist
  b += (size_t)passes * RADIX * 4;  // bin_base
  b = (b + 255) & ~(size_t)255;
  b += (size_t)RADIX * tiles * 4;   // tile counts / offsets
  return b + 256;
}

__host__ inline SortScratch carve_scratch(void* base, long long n, int passes) {
  char* p = (char*)(((uintptr_t)base + 255) & ~(uintptr_t)255);
  SortScratch s;
  s.hist = (unsigned*)p;
  p += (size_t)passes * RADIX * 4;
  s.bin_base = (unsigned*)p;
  p += (size_t)passes * RADIX * 4;
  s.zero_bytes = (size_t)passes * RADIX * 4;
  p = (char*)(((uintptr_t)p + 255) & ~(uintptr_t)255);
  s.counts = (unsigned*)p;
  (void)n;
  return s;
}

// Sorts n pairs by the low `passes*8` key bits.  Buffers ping-pong:
// pass 0 reads (k[0],v[0]) and writes (k[1],v[1]), pass 1 the reverse, ...
// Returns the index (0/1) of the buffer pair that holds the result.
// vals may be null (keys only).  With n_dev non-null the count is read on
// the device (at most n, which sizes the grids and the scratch).
// With `ranges` (and n_dev null) the last pass also writes, for every key
// value below range_keys, its [start, end) in the sorted output into the
// zero-initialised int2 array `ranges` ((0, 0) for absent keys).  `err` is
// kept for the callers' error plumbing; no step of the sort waits on
// another tile, so none can time out.
__host__ inline int sort_pairs(unsigned* k[2], unsigned* v[2], long long n, const int* n_dev, int passes,
                               void* scratch, long long* err, cudaStream_t stream, int* ranges = nullptr,
                               int range_keys = 0) {
  (void)err;
  if ((n <= 1 && !n_dev) || n <= 0 || passes == 0) return 0;
  SortScratch s = carve_scratch(scratch, n, passes);
  cudaMemsetAsync(s.hist, 0, s.zero_bytes, stream);
  const int hist_blocks = (int)std::min<long long>(148 * 4, (n + THREADS * 8 - 1) / (THREADS * 8));
  histogram_kernel<<<std::max(hist_blocks, 1), THREADS, 0, stream>>>(k[0], (int)n, n_dev, passes, s.hist);
  bin_base_kernel<<<passes, THREADS, 0, stream>>>(s.hist, s.bin_base);
  const int tiles = num_tiles(n);
  int cur = 0;
  for (int p = 0; p < passes; ++p) {
    int* rg = (p == passes - 1 && !n_dev) ? ranges : nullptr;
    tile_count_kernel<<<tiles, THREADS, 0, stream>>>(k[cur], (int)n, n_dev, p * RADIX_BITS, s.counts, tiles);
    tile_offset_kernel<<<RADIX, THREADS, 0, stream>>>(s.counts, tiles, s.bin_base + p * RADIX);
    if (v[0]) {
      scatter_kernel<true><<<tiles, THREADS, 0, stream>>>(k[cur], v[cur], k[cur ^ 1], v[cur ^ 1], (int)n, n_dev,
                                                          p * RADIX_BITS, s.counts, tiles, rg, range_keys);
    } else {
      scatter_kernel<false><<<tiles, THREADS, 0, stream>>>(k[cur], nullptr, k[cur ^ 1], nullptr, (int)n, n_dev,
                                                           p * RADIX_BITS, s.counts, tiles, rg, range_keys);
    }
    cur ^= 1;
  }
  if (ranges && !n_dev && range_keys > 0)
    ranges_fixup_kernel<<<(range_keys + 255) / 256, 256, 0, stream>>>(range_keys, (int)n, ranges);
  return cur;
}

}  // namespace
}  // namespace radix
}  // namespace gsb
