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

constexpr int ADAM_THREADS = 256;
constexpr int ADAM_ITEMS = 4;

struct AdamScalars {
  float w1, b2, w2, bc2_sqrt, eps;
  float neg_step[6];  // -lr / bc1 per group
};

__global__ void __launch_bounds__(ADAM_THREADS) adam_kernel(const gsb_adam_args a, AdamScalars s,
                                                           long long total) {
  const long long P = a.P;
  const long long seg_end[5] = {3 * P, 6 * P, 10 * P, 11 * P, total};
  const long long base = ((long long)blockIdx.x * ADAM_THREADS * ADAM_ITEMS) + threadIdx.x;
#pragma unroll
  for (int it = 0; it < ADAM_ITEMS; ++it) {
    const long long e = base + (long long)it * ADAM_THREADS;
    if (e >= total) return;
    int seg = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) seg += e >= seg_end[k];
    const long long local = e - (seg == 0 ? 0 : seg_end[seg - 1]);
    float* p = a.params[seg] + local;
    int group = seg;
    if (seg == 4) group = (local % (3LL * a.sh_coeffs)) < 3 ? 4 : 5;  // SH DC vs the rest
    const float g = a.grad[e];
    float m = a.exp_avg[e];
    float v = a.exp_avg_sq[e];
    m = fmaf(s.w1, g - m, m);
    v = v * s.b2;
    v = fmaf(s.w2 * g, g, v);
    const float denom = sqrtf(v) / s.bc2_sqrt + s.eps;
    *p = fmaf(s.neg_step[group], m / denom, *p);
    a.exp_avg[e] = m;
    a.exp_avg_sq[e] = v;
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
  adam_kernel<<<(unsigned)blocks, ADAM_THREADS, 0, (cudaStream_t)stream>>>(*a, s, total);
  return check_launch("gsb_adam_step");
}

GSB_EXPORT int gsb_densify_stats(int P, const int* radii, float* denom, float* max_radii, void* stream) {
  if (P < 0 || (P > 0 && (!radii || !denom || !max_radii))) {
    set_error("gsb_densify_stats: invalid arguments");
    return GSB_ERR_INVALID;
  }
  if (P == 0) return GSB_OK;
  densify_stats_kernel<<<div_up(P, 256), 256, 0, (cudaStream_t)stream>>>(P, radii, denom, max_radii);
  return check_launch("gsb_densify_stats");
}
