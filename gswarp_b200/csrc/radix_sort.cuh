// radix_sort.cuh -- stable LSD radix sort of (uint32 key, uint32 value) pairs.
//
// Replaces Warp's wp.utils.radix_sort_pairs (called from gswarp
// memory.py:571-600 and knn.py:337-341) with a single-pass-per-digit
// ("onesweep") design for sm_100a:
//   1. one histogram kernel computes the 8-bit digit histograms of every
//      pass in a single read of the keys (warp-aggregated shared atomics);
//   2. a tiny kernel turns them into per-pass bin bases;
//   3. each pass is ONE kernel: a CTA claims the next 3840-key tile through
//      an atomic counter, ranks its keys stably per warp (one ballot per
//      digit bit), publishes its per-digit counts, resolves its global
//      offsets by decoupled look-back over the preceding tiles, stages the
//      tile in digit order in shared memory and writes it out in runs.
// The caller states how many low key bits are significant: every pass takes
// 8 of them except the last, which takes what is left (a 13-bit tile id
// sorts in an 8-bit and a 5-bit pass), and the last pass writes only the
// values (and the key ranges) -- no caller reads the sorted keys.
// Tiles are claimed in launch order, so every tile a CTA waits on belongs to
// a CTA that is already running; each look-back spin is nevertheless bounded
// (SPIN_LIMIT) and reports ERR_LOOKBACK_TIMEOUT instead of hanging.
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
constexpr int LOOKBACK_WINDOW = 4;
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

// Lanes of the warp whose BITS-bit digit d equals this lane's: one ballot
// per bit (cheaper on sm_100a than a match.any over 32 distinct values).
template <int BITS>
__device__ __forceinline__ unsigned digit_peers(unsigned d) {
  unsigned peers = 0xffffffffu;
#pragma unroll
  for (int b = 0; b < BITS; ++b) {
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
                                                            int passes, unsigned last_mask,
                                                            unsigned* __restrict__ hist) {
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
          atomicAdd(&s_hist[warp][p][(kv[it] >> (p * RADIX_BITS)) & (p == passes - 1 ? last_mask : RADIX - 1)],
                    1u);
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

// One pass over the digit of BITS bits at `shift`.  keys_out may be null
// (the last pass: only values and ranges are wanted).
template <int BITS>
__global__ void __launch_bounds__(THREADS, 4) onesweep_kernel(
    const unsigned* __restrict__ keys_in, const unsigned* __restrict__ vals_in,
    unsigned* __restrict__ keys_out, unsigned* __restrict__ vals_out, int n_host,
    const int* __restrict__ n_dev, int shift,
    const unsigned* __restrict__ bin_base, unsigned long long* __restrict__ lookback,
    unsigned* __restrict__ tile_counter, long long* __restrict__ err, int* __restrict__ ranges,
    int range_keys) {
  __shared__ unsigned s_keys[TILE_KEYS];
  __shared__ unsigned s_vals[TILE_KEYS];
  __shared__ unsigned s_warp_hist[WARPS][RADIX];
  __shared__ unsigned s_digit_start[RADIX];
  __shared__ unsigned s_global[RADIX];
  __shared__ unsigned s_scan[WARPS];
  __shared__ int s_tile;

  constexpr unsigned MASK = (1u << BITS) - 1u;
  constexpr int NB = 1 << BITS;  // digits in use; threads tid >= NB own none
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // With a device-side count the grid is sized for the upper bound; CTAs
  // that claim a tile past the end leave (no later tile waits on them).
  const int n = n_dev ? *n_dev : n_host;
  if (tid == 0) s_tile = (int)atomicAdd(tile_counter, 1u);
  for (int i = tid; i < WARPS * RADIX; i += THREADS) (&s_warp_hist[0][0])[i] = 0u;
  __syncthreads();
  const int tile = s_tile;
  if ((long long)tile * TILE_KEYS >= n) return;
  const long long base = (long long)tile * TILE_KEYS + (long long)warp * (ITEMS * 32);

  // Positions past n (only in the last tile) hold the key 0xFFFFFFFF, whose
  // digit is the largest, and are ranked like the others: a warp's missing
  // positions follow all of its valid ones and only later warps have more,
  // so they stage after every valid key of the tile, at [tile_n, TILE_KEYS),
  // where nothing reads them.  Their counts enter the last tile's published
  // totals, which no tile reads (tiles look back only at earlier ones).
  unsigned key[ITEMS], rank[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const long long pos = base + i * 32 + lane;
    key[i] = pos < n ? keys_in[pos] : 0xFFFFFFFFu;
  }
  // Stable warp-local ranking: round i holds 32 consecutive keys.  The
  // lowest lane of each digit group adds the group's size to the warp's
  // counter with a shared atomic and hands the old count to its peers: no
  // read-then-write chain between rounds (shared atomics of one warp to one
  // address take effect in issue order, so rounds keep their order).
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const unsigned d = (key[i] >> shift) & MASK;
    const unsigned peers = digit_peers<BITS>(d);
    const int leader = __ffs(peers) - 1;
    unsigned old = 0;
    if (lane == leader) old = atomicAdd(&s_warp_hist[warp][d], (unsigned)__popc(peers));
    old = __shfl_sync(0xffffffffu, old, leader);
    rank[i] = old + __popc(peers & lt);
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
  unsigned long long* my_slot = lookback + (size_t)tile * RADIX + tid;
  if (tid < NB) st_volatile(my_slot, (tile == 0 ? FLAG_INC : FLAG_AGG) | (unsigned long long)total);
  s_digit_start[tid] = block_exclusive_scan(total, s_scan, nullptr);
  __syncthreads();

  // Stage the tile in digit order (before the look-back, so the key and rank
  // registers are free while it waits); values are read here, not earlier.
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const unsigned d = (key[i] >> shift) & MASK;
    rank[i] += s_digit_start[d] + s_warp_hist[warp][d];
    s_keys[rank[i]] = key[i];
  }
  {
    unsigned val[ITEMS];
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const long long pos = base + i * 32 + lane;
      val[i] = pos < n ? vals_in[pos] : 0u;
    }
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) s_vals[rank[i]] = val[i];
  }

  // Decoupled look-back over a window of LOOKBACK_WINDOW predecessors at a
  // time: the window's status words are loaded together (one memory round
  // trip per window instead of one per tile), then consumed nearest first,
  // adding aggregates until an inclusive prefix is found.  A slot that is not
  // published yet is re-read (bounded) before the walk moves past it.
  unsigned long long excl = 0;
  if (tile > 0 && tid < NB) {
    int t = tile - 1;
    int spins = 0;
    bool done = false;
    while (!done) {
      unsigned long long w[LOOKBACK_WINDOW];
#pragma unroll
      for (int k = 0; k < LOOKBACK_WINDOW; ++k)
        w[k] = t - k >= 0 ? ld_volatile(lookback + (size_t)(t - k) * RADIX + tid) : FLAG_INC;
#pragma unroll
      for (int k = 0; k < LOOKBACK_WINDOW; ++k) {
        if (done) break;
        unsigned long long v = w[k];
        while ((v & ~VALUE_MASK) == 0) {
          if (++spins > SPIN_LIMIT) {
            atomicOr((unsigned long long*)err, (unsigned long long)ERR_LOOKBACK_TIMEOUT);
            break;
          }
          v = ld_volatile(lookback + (size_t)(t - k) * RADIX + tid);
        }
        if ((v & ~VALUE_MASK) == 0) {  // timed out: give up, error already flagged
          done = true;
          break;
        }
        if (t - k >= 0) excl += v & VALUE_MASK;
        if ((v & ~VALUE_MASK) == FLAG_INC || t - k <= 0) done = true;
      }
      t -= LOOKBACK_WINDOW;
    }
    st_volatile(my_slot, FLAG_INC | (excl + total));
  }
  // staged position j of digit d goes to s_global[d] + j (unsigned wrap-around)
  s_global[tid] = bin_base[tid] + (unsigned)excl - s_digit_start[tid];
  __syncthreads();
  const long long tile_base = (long long)tile * TILE_KEYS;
  const int tile_n = (int)min((long long)TILE_KEYS, (long long)n - tile_base);
  for (int j = tid; j < tile_n; j += THREADS) {
    const unsigned k = s_keys[j];
    const unsigned d = (k >> shift) & MASK;
    const unsigned dst = s_global[d] + (unsigned)j;
    // dst < n whenever the histogram and look-back agree; the test keeps a
    // timed-out look-back (flagged above) from writing out of bounds.
    if (dst < (unsigned)n) {
      if (keys_out) keys_out[dst] = k;
      vals_out[dst] = s_vals[j];
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
  unsigned* hist;                  // passes*256
  unsigned* bin_base;              // passes*256
  unsigned* counters;              // passes
  unsigned long long* lookback;    // passes*tiles*256
  size_t zero_bytes;               // bytes to clear from `hist` on
};

__host__ inline int num_tiles(long long n) { return (int)((n + TILE_KEYS - 1) / TILE_KEYS); }

__host__ inline size_t scratch_bytes(long long n, int passes) {
  const size_t tiles = (size_t)num_tiles(n > 0 ? n : 1);
  size_t b = 0;
  b += (size_t)passes * RADIX * 4;   // hist
  b += (size_t)passes * RADIX * 4;   // bin_base
  b += 256;                          // counters (padded)
  b = (b + 255) & ~(size_t)255;
  b += (size_t)passes * tiles * RADIX * 8;
  return b + 256;
}

__host__ inline SortScratch carve_scratch(void* base, long long n, int passes) {
  const size_t tiles = (size_t)num_tiles(n > 0 ? n : 1);
  char* p = (char*)(((uintptr_t)base + 255) & ~(uintptr_t)255);
  SortScratch s;
  char* start = p;
  s.hist = (unsigned*)p;
  p += (size_t)passes * RADIX * 4;
  s.bin_base = (unsigned*)p;
  p += (size_t)passes * RADIX * 4;
  s.counters = (unsigned*)p;
  p += 256;
  p = (char*)(((uintptr_t)p + 255) & ~(uintptr_t)255);
  s.lookback = (unsigned long long*)p;
  p += (size_t)passes * tiles * RADIX * 8;
  s.zero_bytes = (size_t)(p - start);
  return s;
}

// Passes needed for keys of `key_bits` significant low bits.
__host__ inline int passes_for_bits(int key_bits) { return (key_bits + RADIX_BITS - 1) / RADIX_BITS; }

template <int BITS>
__host__ inline void launch_pass(int tiles, cudaStream_t stream, const unsigned* ki, const unsigned* vi,
                                 unsigned* ko, unsigned* vo, int n, const int* n_dev, int shift,
                                 const unsigned* base, unsigned long long* lb, unsigned* counter, long long* err,
                                 int* rg, int range_keys) {
  onesweep_kernel<BITS><<<tiles, THREADS, 0, stream>>>(ki, vi, ko, vo, n, n_dev, shift, base, lb, counter, err, rg,
                                                       range_keys);
}

// Sorts n pairs by the low `key_bits` (1..32) key bits (higher bits are
// ignored).  Buffers ping-pong: pass 0 reads (k[0],v[0]) and writes
// (k[1],v[1]), pass 1 the reverse, ...  Returns the index (0/1) of the
// buffer pair that holds the sorted values; the last pass does not write
// keys, so the sorted keys are not kept.  With n_dev non-null the count is read on
// the device (at most n, which sizes the grids and the scratch).
// With `ranges` (and n_dev null) the last pass also writes, for every key
// value below range_keys, its [start, end) in the sorted output into the
// zero-initialised int2 array `ranges` ((0, 0) for absent keys).
__host__ inline int sort_pairs(unsigned* k[2], unsigned* v[2], long long n, const int* n_dev, int key_bits,
                               void* scratch, long long* err, cudaStream_t stream, int* ranges = nullptr,
                               int range_keys = 0) {
  const int passes = passes_for_bits(key_bits);
  if ((n <= 1 && !n_dev) || n <= 0 || passes == 0) return 0;
  const int last_bits = key_bits - RADIX_BITS * (passes - 1);
  SortScratch s = carve_scratch(scratch, n, passes);
  cudaMemsetAsync(s.hist, 0, s.zero_bytes, stream);
  const int hist_blocks = (int)std::min<long long>(148 * 4, (n + THREADS * 8 - 1) / (THREADS * 8));
  histogram_kernel<<<std::max(hist_blocks, 1), THREADS, 0, stream>>>(k[0], (int)n, n_dev, passes,
                                                                      (1u << last_bits) - 1u, s.hist);
  bin_base_kernel<<<passes, THREADS, 0, stream>>>(s.hist, s.bin_base);
  const int tiles = num_tiles(n);
  int cur = 0;
  for (int p = 0; p < passes; ++p) {
    unsigned long long* lb = s.lookback + (size_t)p * tiles * RADIX;
    const bool last = p == passes - 1;
    int* rg = (last && !n_dev) ? ranges : nullptr;
    unsigned* ko = last ? nullptr : k[cur ^ 1];
    const unsigned* vi = v[cur];
    unsigned* vo = v[cur ^ 1];
    const int bits = last ? last_bits : RADIX_BITS;
    const unsigned* base = s.bin_base + p * RADIX;
    const int sh = p * RADIX_BITS;
    switch (bits) {
      case 1: launch_pass<1>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      case 2: launch_pass<2>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      case 3: launch_pass<3>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      case 4: launch_pass<4>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      case 5: launch_pass<5>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      case 6: launch_pass<6>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      case 7: launch_pass<7>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
      default: launch_pass<8>(tiles, stream, k[cur], vi, ko, vo, (int)n, n_dev, sh, base, lb, s.counters + p, err, rg, range_keys); break;
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
