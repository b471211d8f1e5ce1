"""fused_ssim autograd contracts, after the reference's own contract tests
(tests/test_fused_ssim_cuda_contracts.py:38-186): forwards that are alive at
the same time keep their own backward state, a non-default stream and two
streams give the isolated results, retain_graph repeats the backward, and a
returned gradient is not overwritten by a later call."""

import pytest
import torch

import gswarp_b200 as gs
from gswarp_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _pair(seed, shape=(1, 3, 48, 64)):
    a, b = wl.config3_images(seed=seed, shape=shape)
    return a.cuda(), b.cuda()


def _isolated(img1, img2):
    x = img1.clone().requires_grad_(True)
    loss = gs.fused_ssim(x, img2)
    loss.backward()
    torch.cuda.synchronize()
    return loss.detach().clone(), x.grad.clone()


def test_multiple_live_forwards_keep_independent_backward_state(cuda):
    (a1, b1), (a2, b2) = _pair(1), _pair(2)
    ref1, ref2 = _isolated(a1, b1), _isolated(a2, b2)
    x1, x2 = a1.clone().requires_grad_(True), a2.clone().requires_grad_(True)
    l1 = gs.fused_ssim(x1, b1)
    l2 = gs.fused_ssim(x2, b2)  # both graphs alive before either backward
    l2.backward()
    l1.backward()
    torch.cuda.synchronize()
    assert torch.equal(l1.detach(), ref1[0]) and torch.equal(l2.detach(), ref2[0])
    assert torch.equal(x1.grad, ref1[1]) and torch.equal(x2.grad, ref2[1])


def test_non_default_stream(cuda):
    a, b = _pair(3)
    ref = _isolated(a, b)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        x = a.clone().requires_grad_(True)
        loss = gs.fused_ssim(x, b)
        loss.backward()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert torch.equal(loss.detach(), ref[0]) and torch.equal(x.grad, ref[1])


def test_two_streams_match_isolated_gradients(cuda):
    pairs = [_pair(4, (2, 3, 96, 80)), _pair(5, (2, 3, 96, 80))]
    refs = [_isolated(a, b) for a, b in pairs]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    out = []
    for s, (a, b) in zip(streams, pairs):
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            x = a.clone().requires_grad_(True)
            loss = gs.fused_ssim(x, b)
            loss.backward()
            out.append((loss, x))
    for s in streams:
        torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for (loss, x), (rl, rg) in zip(out, refs):
        assert torch.equal(loss.detach(), rl) and torch.equal(x.grad, rg)


def test_retain_graph_repeats_backward(cuda):
    a, b = _pair(6)
    x = a.clone().requires_grad_(True)
    loss = gs.fused_ssim(x, b)
    loss.backward(retain_graph=True)
    g1 = x.grad.clone()
    x.grad = None
    loss.backward()
    torch.cuda.synchronize()
    assert torch.equal(x.grad, g1)


def test_later_call_does_not_overwrite_returned_gradient(cuda):
    a, b = _pair(7)
    c, d = _pair(8)
    x = a.clone().requires_grad_(True)
    (g,) = torch.autograd.grad(gs.fused_ssim(x, b), x)
    kept = g.clone()
    y = c.clone().requires_grad_(True)
    gs.fused_ssim(y, d).backward()  # same shapes: a reused buffer would land in g
    torch.cuda.synchronize()
    assert torch.equal(g, kept)
