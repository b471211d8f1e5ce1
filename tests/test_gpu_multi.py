"""Two-GPU training step (needs at least two GPUs; skipped otherwise).

Two NCCL ranks, each rendering its own views of the same scene.  The
multi-view-SH step all-reduces the blocks complete after the last view while
the SH backward runs, the SH rows range by range and the means last; the
range-ordered variant computes the per-Gaussian backward one Gaussian range
at a time and all-reduces each finished range while the next one is
computed.  Both must equal (up to the render backward's atomic summation
order) the per-view-SH step's single all-reduce of the whole buffer, and the
sum of the ranks' local gradients."""

import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _close(a: torch.Tensor, b: torch.Tensor, sizes) -> None:
    off = 0
    for k in sizes:
        x, y = a[off:off + k], b[off:off + k]
        assert float((x - y).norm()) <= 1e-4 * float(y.norm()) + 1e-7, off
        off += k


def _worker(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist

    import gswarp_b200 as gs
    from gswarp_b200 import workloads as wl
    from gswarp_b200.training import FusedViewStep

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        singles = [dist.new_group(ranks=[r]) for r in range(world)]
        sc = wl.config2_scene(seed=5, n=30_000)
        cams = wl.ring_views(2 * world, seed=5, width=320, height=192)[2 * rank: 2 * rank + 2]
        params = [t.to(dev).contiguous() for t in (sc.means, sc.scales, sc.rotations, sc.opacities, sc.sh)]
        bg = torch.zeros(3, device=dev)
        settings = [gs.GaussianRasterizationSettings(
            image_height=v.height, image_width=v.width, tanfovx=v.tanfovx, tanfovy=v.tanfovy, bg=bg,
            scale_modifier=1.0, viewmatrix=v.viewmatrix.to(dev), projmatrix=v.projmatrix.to(dev), sh_degree=3,
            campos=v.campos.to(dev), prefiltered=False) for v in cams]
        targets = [wl.target_image(100 + 2 * rank + i, 192, 320).to(dev) for i in range(2)]
        sizes = [p.numel() for p in params]

        overlapped = FusedViewStep([p.clone() for p in params], settings, batch_sh=True)
        overlapped.sh_reduce_chunks = 3
        overlapped.step(targets)
        ranged = FusedViewStep([p.clone() for p in params], settings, batch_sh=True)
        ranged.range_backward = True
        ranged.backward_chunks = 3
        ranged.step(targets)
        plain = FusedViewStep([p.clone() for p in params], settings, batch_sh=False)
        plain.step(targets)
        local = FusedViewStep([p.clone() for p in params], settings, batch_sh=True, group=singles[rank])
        local.step(targets)
        summed = local.grads.flat.clone()
        dist.all_reduce(summed)
        torch.cuda.synchronize()
        got = overlapped.grads.flat
        assert float(got.abs().sum()) > 0
        assert float((got - local.grads.flat).norm()) > 1e-3 * float(got.norm())  # the other rank contributed
        _close(got, plain.grads.flat, sizes)
        _close(got, summed, sizes)
        _close(ranged.grads.flat, summed, sizes)
        # every rank holds the same reduced buffer
        first = got.clone()
        dist.broadcast(first, src=0)
        assert torch.equal(first, got)
        assert not bool(overlapped._grad_colors.any())
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_rank_step_overlapped_reduction_matches_single_all_reduce():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.multiprocessing.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
