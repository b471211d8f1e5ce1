// peaks.cu -- measurement microkernels for the compute roofline of the
// render kernels: FP32 fused multiply-add throughput (packed f32x2, the form
// the render kernels issue) and MUFU ex2 throughput.  bench.py times them
// with CUDA events and divides the work below by the time.
//
// Each thread runs CHAINS independent dependency chains so the pipes, not
// latency, bound the rate; the results feed a data-dependent store so the
// compiler keeps every operation.
#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int PEAK_THREADS = 256;
constexpr int CHAINS = 8;

// Per thread and iteration: CHAINS packed FMAs = CHAINS * 2 FMA = CHAINS * 4 FLOP.
__global__ void __launch_bounds__(PEAK_THREADS) fp32_peak_kernel(int iters, float seed, float* out) {
  float2 a[CHAINS];
#pragma unroll
  for (int k = 0; k < CHAINS; ++k) a[k] = make_float2(seed + threadIdx.x * 1e-3f + k, seed - k * 1e-3f);
  const float2 m = make_float2(0.9999999f, 0.9999998f);
  const float2 c = make_float2(1.0e-7f, 2.0e-7f);
  // unrolled so the loop counter and branch are a small share of the issue slots
#pragma unroll 16
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < CHAINS; ++k) a[k] = __ffma2_rn(a[k], m, c);
  }
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < CHAINS; ++k) s += a[k].x + a[k].y;
  if (s == 1234.5678f) out[blockIdx.x] = s;  // never true for these inputs; keeps the chains live
}

__device__ __forceinline__ float ex2_approx_ftz(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Per thread and iteration: CHAINS ex2 evaluations (x -> 2^-x stays in (0.5, 1]).
__global__ void __launch_bounds__(PEAK_THREADS) ex2_peak_kernel(int iters, float seed, float* out) {
  float a[CHAINS];
#pragma unroll
  for (int k = 0; k < CHAINS; ++k) a[k] = seed + threadIdx.x * 1e-4f + k * 1e-3f;
#pragma unroll 16
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < CHAINS; ++k) a[k] = ex2_approx_ftz(-a[k]);
  }
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < CHAINS; ++k) s += a[k];
  if (s == 1234.5678f) out[blockIdx.x] = s;
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_peak_fp32(int blocks, int iters, float* out, void* stream) {
  if (blocks <= 0 || iters <= 0 || !out) {
    set_error("gsb_peak_fp32: invalid arguments");
    return GSB_ERR_INVALID;
  }
  fp32_peak_kernel<<<blocks, PEAK_THREADS, 0, (cudaStream_t)stream>>>(iters, 0.5f, out);
  return check_launch("fp32_peak_kernel");
}

GSB_EXPORT int gsb_peak_ex2(int blocks, int iters, float* out, void* stream) {
  if (blocks <= 0 || iters <= 0 || !out) {
    set_error("gsb_peak_ex2: invalid arguments");
    return GSB_ERR_INVALID;
  }
  ex2_peak_kernel<<<blocks, PEAK_THREADS, 0, (cudaStream_t)stream>>>(iters, 0.5f, out);
  return check_launch("ex2_peak_kernel");
}

GSB_EXPORT long long gsb_peak_work(int which, int blocks, int iters) {
  // FLOP (which = 0) or ex2 evaluations (which = 1) of one launch
  const long long per_thread_iter = which == 0 ? (long long)CHAINS * 4 : (long long)CHAINS;
  return (long long)blocks * PEAK_THREADS * iters * per_thread_iter;
}
