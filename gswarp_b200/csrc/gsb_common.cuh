// gsb_common.cuh -- shared device helpers and host-side error plumbing for
// libgsb200 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/gsb200.h"
#include "gsb_launch.cuh"

#define GSB_EXPORT extern "C" __attribute__((visibility("default")))

namespace gsb {

constexpr int BLOCK_X = 16;
constexpr int BLOCK_Y = 16;
constexpr int TILE_PIXELS = BLOCK_X * BLOCK_Y;

// Error bits OR-ed into the device error word.
constexpr long long ERR_LOOKBACK_TIMEOUT = 1ll << 0;
constexpr long long ERR_EMIT_MISMATCH = 1ll << 1;

// Bound for every device-side spin (decoupled look-back).  A predecessor
// tile's CTA is always resident when a successor spins on it (tiles are
// claimed in launch order through an atomic counter), so the bound is a
// safety net that turns an impossible hang into an error flag.
constexpr int SPIN_LIMIT = 1 << 24;

void set_error(const char* fmt, ...);
int check_launch(const char* what);

inline int div_up(long long a, long long b) { return (int)((a + b - 1) / b); }

// ---- float helpers matching the reference's min/max/clamp semantics ----
__host__ __device__ __forceinline__ float fmn(float a, float b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ float fmx(float a, float b) { return a > b ? a : b; }
__host__ __device__ __forceinline__ float fclamp(float x, float lo, float hi) {
  return fmn(fmx(x, lo), hi);
}
__host__ __device__ __forceinline__ int imn(int a, int b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int imx(int a, int b) { return a > b ? a : b; }

// Saturating float->int32 truncation (cvt.rzi.s32.f32): the conversion
// Warp's wp.int32() compiles to.
__device__ __forceinline__ int f2i(float x) { return __float2int_rz(x); }

// Correctly rounded binary32 natural log (evaluated through fp64); see the
// AccuTile threshold in gsb_geometry.cuh.
__device__ __forceinline__ float crlogf(float x) { return (float)log((double)x); }

// Fast exp for the render hot loops: ex2.approx on x*log2(e).
__device__ __forceinline__ float fast_exp(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// 16-byte vector reduction into global memory (sm_90+).
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

}  // namespace gsb
