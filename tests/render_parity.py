"""Render parity rules shared by the GPU tests (a helper module of tests/,
not a test file).

The render kernels evaluate exp as ``ex2.approx`` of the exponent in log2
units formed with fused multiply-adds; the oracle (like the reference's
kernel code, which it reproduces bit for bit) uses the C library's ``expf``
of the exponent in the reference's operation order.  For the exponents that
matter (alpha >= 1/255 needs power >= -ln 255) the two differ by about 1e-6
relative at most, so a thresholded decision (exponent sign, alpha >= 1/255,
T*(1-alpha) < 1e-4) whose relative distance from its threshold exceeds
``DECISION_EPS`` is taken the same way by both.  Measured at config 2 full
size (1M Gaussians, 1080p): every pixel that differs had a margin below
7.2e-7, and 0.03% of pixels have a margin below 1e-5.

Forward: every pixel is within rtol 1e-4 / atol 1e-5 on colour, alpha and
depth with an equal n_contrib, unless the oracle's margin for that pixel is
below DECISION_EPS.  There are no other exceptions.

Backward (both sides given the same forward state): each gradient component
is within ``1e-5 + 1e-4 |ref| + 2e-6 * sum|terms| + 8 * 2^-24 * sum|term| * s``;
the third term is the float32 conditioning of a sum whose terms carry the
~1e-6 relative exp difference and are added in another order (warp
reductions and atomics against the oracle's float64 sum), the fourth the
rounding of each term's exponent, whose terms have size s (elongated
Gaussians far from their centre line have large s and a small exponent).  A component may exceed that only by at
most the sum of |terms| it receives from pixels whose backward margin is
below DECISION_EPS (what a decision taken the other way can change); an
excess beyond it is an unexplained outlier and fails.
"""

from __future__ import annotations

import numpy as np

import oracle

DECISION_EPS = 1e-5
# Rounding of the exponent: the kernels form it in log2 units with fused
# multiply-adds, the reference as -(a dx^2 + c dy^2)/2 - b dx dy; each is a few
# roundings of terms of size s = (|a| dx^2 + |c| dy^2)/2 + |b dx dy|, so the
# two exponents may differ by ~eps32 * s and exp(power) relatively by as much.
# A term's allowance is 8 * 2^-24 * s (cond_abs sums |term| * s).
EXP_ROUNDING = 8 * 2.0 ** -24
MAX_FLAGGED_PIXELS = 1e-3  # the rule may excuse at most this fraction of pixels


def forward_inputs(records: np.ndarray, ranges, point_list, bg):
    """Oracle render inputs from the GPU's 48-byte render records."""
    return dict(ranges=ranges, point_list=point_list, xy=records[:, 0:2].copy(), features=records[:, 8:11].copy(),
                depths=records[:, 6].copy(), conic_opacity=np.concatenate([records[:, 2:4], records[:, 4:6]], 1).copy(),
                bg=bg)


def check_forward(W, H, inp, got_color, got_depth, got_alpha, got_nc, compute_depth=True):
    """Returns the oracle's (color, depth, alpha, n_contrib) after checking
    the GPU's against them with the margin rule."""
    col, dep, alp, nc, margin, _ = oracle.render_fwd(W, H, inp["ranges"], inp["point_list"], inp["xy"],
                                                     inp["features"], inp["depths"], inp["conic_opacity"],
                                                     inp["bg"], compute_depth, with_margin=True)
    bad = (np.asarray(got_nc).reshape(H, W) != nc.reshape(H, W))
    for got, ref in ((got_color, col), (got_alpha, alp), (got_depth, dep)):
        g = np.asarray(got).reshape(ref.shape)
        bad |= (np.abs(g - ref) > 1e-5 + 1e-4 * np.abs(ref)).reshape(-1, H, W).any(0)
    flagged = margin < DECISION_EPS
    unexplained = bad & ~flagged
    assert not unexplained.any(), (
        f"{int(unexplained.sum())} pixels outside tolerance with a decision margin >= {DECISION_EPS}: "
        f"first at (y, x) = {tuple(np.argwhere(unexplained)[0])}")
    assert flagged.mean() <= MAX_FLAGGED_PIXELS, f"{flagged.mean():.2e} of pixels near a threshold"
    return col, dep, alp, nc


def check_backward(W, H, P, inp, out_alpha, n_contrib, grad_color, grad_depth, grad_alpha, got, compute_depth=True):
    """``got``: (P, 10) GPU gradients ordered xy(2), depth, conic_opacity(4),
    rgb(3).  Returns the oracle result dict."""
    ref = oracle.render_bwd(W, H, P, inp["ranges"], inp["point_list"], inp["xy"], inp["features"], inp["depths"],
                            inp["conic_opacity"], inp["bg"], out_alpha, n_contrib, grad_color, grad_depth,
                            grad_alpha, compute_depth, with_abs=True, with_margin=True, flag_eps=DECISION_EPS)
    want = np.concatenate([ref["grad_xy"], ref["grad_depth"][:, None], ref["grad_conic_opacity"], ref["grad_rgb"]],
                          1).astype(np.float64)
    tol = 1e-5 + 1e-4 * np.abs(want) + 2e-6 * ref["abs"] + EXP_ROUNDING * ref["cond_abs"]
    excess = np.abs(np.asarray(got, np.float64) - want) - tol
    unexplained = excess > ref["flagged_abs"]
    assert not unexplained.any(), (
        f"{int(unexplained.sum())} gradient entries ({int(unexplained.any(1).sum())} Gaussians) outside tolerance "
        f"beyond what near-threshold pixels contribute; first Gaussian {int(np.argwhere(unexplained)[0][0])}")
    assert (ref["margin"] < DECISION_EPS).mean() <= MAX_FLAGGED_PIXELS
    return ref


def gpu_grads(grad_acc: np.ndarray) -> np.ndarray:
    """(P, 10) from the (P, 12) render-gradient accumulator."""
    return np.concatenate([grad_acc[:, 0:3], grad_acc[:, 4:8], grad_acc[:, 8:11]], 1)
