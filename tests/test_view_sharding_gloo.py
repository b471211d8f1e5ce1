"""Host logic of the multi-view data-parallel step, on CPU gloo ranks:
view sharding, in-place gradient accumulation into the flat buffer, the sum
all-reduce across ranks, max-over-ranks timing, and failure propagation
(a rank that dies before the collective makes its peers raise after the
process-group timeout instead of hanging)."""

import json
import multiprocessing as mp
import os
import socket
import tempfile
import time
from datetime import timedelta

import pytest
import torch

from gswarp_b200.view_sharding import GradientBuffer, ViewShardedStep, max_over_ranks, shard_views

N_ITEMS = 37
VIEWS = 8


def _params(seed=0):
    g = torch.Generator().manual_seed(seed)
    shapes = [(N_ITEMS, 3), (N_ITEMS, 3), (N_ITEMS, 4), (N_ITEMS, 1), (N_ITEMS, 16, 3)]
    return [torch.randn(*s, generator=g).requires_grad_(True) for s in shapes]


def _view_weights(view):
    g = torch.Generator().manual_seed(1000 + view)
    shapes = [(N_ITEMS, 3), (N_ITEMS, 3), (N_ITEMS, 4), (N_ITEMS, 1), (N_ITEMS, 16, 3)]
    return [torch.randn(*s, generator=g) for s in shapes]


def _view_loss(params, view):
    # d loss / d p = w_view + 2 * p * 0.01 : known per-view gradients
    ws = _view_weights(view)
    return sum((p * w).sum() + 0.01 * (p * p).sum() for p, w in zip(params, ws))


def test_shard_views_partitions_all_views():
    for views in (8, 16, 64, 7, 1):
        for world in (1, 2, 4, 8):
            parts = [list(shard_views(views, world, r)) for r in range(world)]
            flat = [i for p in parts for i in p]
            assert flat == list(range(views))
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_views(8, 2, 2)


def test_backward_ranges_and_slices_cover_the_buffer_once():
    """The multi-view step's range-ordered backward: Gaussian ranges in
    order, covering [0, P) once, and per range one slice per SoA block of
    the flat gradient buffer; over all ranges the slices are disjoint and
    cover the buffer exactly."""
    from gswarp_b200.training import backward_ranges, range_slices

    blocks = (3, 3, 4, 1, 48)
    for P in (1, 2, 37, 1000, 6_000_001):
        for chunks in (1, 3, 8, 64):
            ranges = backward_ranges(P, chunks)
            assert len(ranges) == max(1, min(chunks, P))
            assert ranges[0][0] == 0 and ranges[-1][1] == P
            assert all(r0[1] == r1[0] and r0[0] < r0[1] for r0, r1 in zip(ranges, ranges[1:]))
            slices = sorted(sl for b, e in ranges for sl in range_slices(P, blocks, b, e))
            assert slices[0][0] == 0 and slices[-1][1] == 59 * P
            assert all(a[1] == b[0] for a, b in zip(slices, slices[1:]))
    assert backward_ranges(0, 8) == []
    assert range_slices(10, blocks, 2, 5) == [(6, 15), (36, 45), (68, 80), (102, 105), (206, 350)]


def test_gradient_buffer_accumulates_in_place():
    params = _params()
    step = ViewShardedStep(params, range(VIEWS), lambda v: _view_loss(params, v))
    step.step()
    flat = step.grads.flat
    assert flat.numel() == N_ITEMS * 59
    assert step.grads.floats_per_item == 59
    expect = torch.cat([sum(ws[k] for ws in map(_view_weights, range(VIEWS))).reshape(-1)
                        + VIEWS * 0.02 * params[k].detach().reshape(-1) for k in range(5)])
    torch.testing.assert_close(flat, expect, rtol=1e-5, atol=1e-5)
    for p, v in zip(params, step.grads.views):
        assert p.grad.data_ptr() == v.data_ptr()
    step.step()  # zeroed and re-accumulated, not doubled
    torch.testing.assert_close(step.grads.flat, expect, rtol=1e-5, atol=1e-5)


def test_first_view_without_a_gradient_leaves_a_zero_block():
    """The first view's gradients are copied into the buffer: a parameter the
    first view does not use gets a zero block (no stale values from the
    previous step), and later views add into the attached blocks."""
    params = _params()

    def loss(v):
        full = _view_loss(params, v)
        return full if v > 0 else (params[0] * 2.0).sum()

    step = ViewShardedStep(params, range(3), loss)
    step.grads.flat.fill_(7.0)  # stale contents must not survive the step
    step.step()
    expect = []
    for k in range(5):
        e = sum(_view_weights(v)[k] for v in (1, 2)).reshape(-1) + 2 * 0.02 * params[k].detach().reshape(-1)
        if k == 0:
            e = e + 2.0
        expect.append(e)
    torch.testing.assert_close(step.grads.flat, torch.cat(expect), rtol=1e-5, atol=1e-5)
    for p, v in zip(params, step.grads.views):
        assert p.grad.data_ptr() == v.data_ptr()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    result = {"rank": rank}
    try:
        torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                             timeout=timedelta(seconds=4))
        params = _params()
        mine = list(shard_views(VIEWS, world, rank))
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # dies before the collective
        step = ViewShardedStep(params, mine, lambda v: _view_loss(params, v))
        t0 = time.perf_counter()
        step.step()
        ms = (time.perf_counter() - t0) * 1000.0 + rank  # distinct per rank
        result["max_ms"] = max_over_ranks(ms)
        result["my_ms"] = ms
        result["flat"] = step.grads.flat.tolist()
        result["views"] = mine
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except SystemExit:
        raise
    except Exception as exc:  # noqa: BLE001 - report any collective failure to the parent
        result["error"] = f"{type(exc).__name__}: {exc}"[:300]
    with open(out_path, "w") as f:
        json.dump(result, f)


def _run(world, mode):
    port = _free_port()
    ctx = mp.get_context("spawn")
    tmp = tempfile.mkdtemp()
    paths = [os.path.join(tmp, f"r{r}.json") for r in range(world)]
    procs = [ctx.Process(target=_worker, args=(r, world, port, paths[r], mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank hung")
    out = []
    for p in paths:
        out.append(json.load(open(p)) if os.path.exists(p) else None)
    return out, [p.exitcode for p in procs]


def test_two_rank_all_reduce_matches_single_process():
    results, codes = _run(2, "ok")
    assert codes == [0, 0]
    params = _params()
    single = ViewShardedStep(params, range(VIEWS), lambda v: _view_loss(params, v))
    single.step()
    ref = single.grads.flat
    assert sorted(results[0]["views"] + results[1]["views"]) == list(range(VIEWS))
    for r in results:
        assert "error" not in r, r.get("error")
        torch.testing.assert_close(torch.tensor(r["flat"]), ref, rtol=1e-5, atol=1e-4)
        assert r["max_ms"] == pytest.approx(max(x["my_ms"] for x in results))


def test_dead_rank_makes_peers_raise_instead_of_hanging():
    t0 = time.time()
    results, codes = _run(2, "fail")
    assert codes[1] == 3
    assert results[0] is not None and "error" in results[0]
    assert time.time() - t0 < 80
