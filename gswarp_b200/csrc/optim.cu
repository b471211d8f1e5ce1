// optim.cu -- fused Adam step over the flat gradient buffer, and the
// densification statistics of the 3DGS training loop.
//
// The training step leaves every per-Gaussian gradient in one flat fp32
// buffer [means 3P | scales 3P | rotations 4P | opacities P | SH 3KP]
// (summed over the step's views and, on several GPUs, all-reduced).  The
// optimizer that follows is the other HBM-bound per-Gaussian pass of a 3DGS
// iteration: torch.optim.Adam over the six 3DGS parameter groups (means,
// scales, rotations, opacities, SH DC, SH rest; each with its own learning
// rate) costs one foreach kernel per arithmetic step per group.  Here it is
// one pass: each element's parameter, gradient and two moments are read
// once and written once (28 bytes), with the arithmetic of torch's Adam
// (torch/optim/adam.py, weight_decay 0, no amsgrad): m = lerp(m, g, 1-b1),
// v = v*b2 + (1-b2)*g*g, p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps).
//
// Densification statistics (3DGS add_densification_stats and the
// max_radii2D update): for every Gaussian with a radius this view,
// denom += 1 and max_radii = max(max_radii, radius); the accumulated norm of
// the screen-space gradient is added by preprocess backward, which holds it.
#include <cmath>

#include "gsb_common.cuh"

namespace gsb {
namespace {

constexpr int ADAM_THREADS = launch::ADAM;
constexpr int ADAM_ITEMS = 4;

struct AdamScalars {
  float w1, b2, w2, bc2_sqrt, eps;
  float neg_step[6];  // -lr / bc1 per group
};

// 32-bit element indices (the host checks that the buffer holds fewer than
// 2^32 elements); each thread handles ADAM_ITEMS elements ADAM_THREADS apart
// so every load and store instruction of a warp is one coalesced run, and
// all of a thread's loads are issued before its arithmetic.
__global__ void __launch_bounds__(ADAM_THREADS) adam_kernel(const gsb_adam_args a, AdamScalars s,
                                                           unsigned total) {
  const unsigned P = (unsigned)a.P;
  const unsigned e1 = 3u * P, e2 = 6u * P, e3 = 10u * P, e4 = 11u * P;
  const unsigned row = 3u * (unsigned)a.sh_coeffs;
  const unsigned base = blockIdx.x * (ADAM_THREADS * ADAM_ITEMS) + threadIdx.x;
  float g[ADAM_ITEMS], m[ADAM_ITEMS], v[ADAM_ITEMS], pv[ADAM_ITEMS];
  float* pp[ADAM_ITEMS];
  int grp[ADAM_ITEMS];
#pragma unroll
  for (int it = 0; it < ADAM_ITEMS; ++it) {
    const unsigned e = base + it * ADAM_THREADS;
    pp[it] = nullptr;
    grp[it] = 0;
    if (e < total) {
      unsigned local;
      int seg;
      if (e < e1) { seg = 0; local = e; }
      else if (e < e2) { seg = 1; local = e - e1; }
      else if (e < e3) { seg = 2; local = e - e2; }
      else if (e < e4) { seg = 3; local = e - e3; }
      else { seg = 4; local = e - e4; }
      grp[it] = seg == 4 ? (local % row < 3u ? 4 : 5) : seg;  // SH DC (coefficient 0) vs the rest
      pp[it] = a.params[seg] + local;
      g[it] = a.grad[e];
      m[it] = a.exp_avg[e];
      v[it] = a.exp_avg_sq[e];
      pv[it] = *pp[it];
    }
  }
#pragma unroll
  for (int it = 0; it < ADAM_ITEMS; ++it) {
    const unsigned e = base + it * ADAM_THREADS;
    if (!pp[it]) continue;
    float mm = fmaf(s.w1, g[it] - m[it], m[it]);
    float vv = v[it] * s.b2;
    vv = fmaf(s.w2 * g[it], g[it], vv);
    const float denom = sqrtf(vv) / s.bc2_sqrt + s.eps;
    *pp[it] = fmaf(s.neg_step[grp[it]], mm / denom, pv[it]);
    a.exp_avg[e] = mm;
    a.exp_avg_sq[e] = vv;
  }
}

__global__ void densify_stats_kernel(int P, const int* __restrict__ radii, float* __restrict__ denom,
                                     float* __restrict__ max_radii) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const int r = radii[i];
  if (r > 0) {
    denom[i] += 1.0f;
    max_radii[i] = fmaxf(max_radii[i], (float)r);
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

GSB_EXPORT int gsb_adam_step(const gsb_adam_args* a, void* stream) {
  if (!a || a->P < 0 || a->sh_coeffs <= 0 || a->step < 1 || !a->grad || !a->exp_avg || !a->exp_avg_sq) {
    set_error("gsb_adam_step: invalid arguments");
    return GSB_ERR_INVALID;
  }
  for (int k = 0; k < 5; ++k)
    if (!a->params[k]) {
      set_error("gsb_adam_step: null parameter pointer");
      return GSB_ERR_INVALID;
    }
  if (a->P == 0) return GSB_OK;
  const long long total = (long long)a->P * (11 + 3LL * a->sh_coeffs);
  if (total >= (1ll << 32) - (long long)ADAM_THREADS * ADAM_ITEMS) {
    set_error("gsb_adam_step: the flat buffer must hold fewer than 2^32 elements");
    return GSB_ERR_INVALID;
  }
  AdamScalars s;
  const double b1 = a->beta1, b2 = a->beta2;
  const double bc1 = 1.0 - std::pow(b1, (double)a->step);
  const double bc2 = 1.0 - std::pow(b2, (double)a->step);
  s.w1 = (float)(1.0 - b1);
  s.b2 = (float)b2;
  s.w2 = (float)(1.0 - b2);
  s.bc2_sqrt = (float)std::sqrt(bc2);
  s.eps = (float)a->eps;
  for (int k = 0; k < 6; ++k) s.neg_step[k] = (float)(-(a->lr[k] / bc1));
  const long long per_block = (long long)ADAM_THREADS * ADAM_ITEMS;
  const long long blocks = (total + per_block - 1) / per_block;
  adam_kernel<<<(unsigned)blocks, ADAM_THREADS, 0, (cudaStream_t)stream>>>(*a, s, (unsigned)total);
  return check_launch("gsb_adam_step");
}

GSB_EXPORT int gsb_densify_stats(int P, const int* radii, float* denom, float* max_radii, void* stream) {
  if (P < 0 || (P > 0 && (!radii || !denom || !max_radii))) {
    set_error("gsb_densify_stats: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (P == 0) return GSB_OK;
  densify_stats_kernel<<<div_up(P, ADAM_THREADS), ADAM_THREADS, 0, (cudaStream_t)stream>>>(P, radii, denom, max_radii);
  return check_launch("gsb_densify_stats");
}
