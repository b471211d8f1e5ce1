"""Golden vectors from gswarp's own kernel code.

    python tests/golden/make_kernel_golden.py /path/to/gswarp  [names...]

gswarp's kernels are Warp (``@wp.kernel``) Python functions, and
``warp-lang`` is not installed here, so this script loads gswarp's kernel
modules under the pure-Python stand-in ``warp_standin.py`` and runs the
kernel bodies themselves on small seeded inputs, with the launch sequence of
gswarp's host code (cited per stage below).  It writes ``kernels_*.npz`` next
to itself: the inputs and every stage's outputs.  ``tests/test_golden_kernels.py``
requires the CPU oracle to reproduce them, and ``tests/test_gpu_golden.py``
the CUDA kernels.

What is the reference's own code here: every ``@wp.kernel`` / ``@wp.func``
body (preprocess, SH colour, coverage count, depth-sort payload, emit, tile
ranges, render forward and backward, SH backward, preprocess backward, SSIM
passes, KNN).  What is restated: the host glue between launches (buffer
shapes, the stable radix sorts as numpy stable argsorts, the inclusive scan,
the mean of the SSIM map), Warp's runtime (warp_standin.py), and the
transcendental functions (the C library's expf; the correctly rounded log).
"""

from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(ROOT))

import warp_standin as ws  # noqa: E402

F32 = np.float32
BLOCK = 16


def load_reference(root: Path) -> dict:
    ws.install()
    base = root / "gswarp" / "_internal" / "backends" / "warp"
    ws.package("gsref", root / "gswarp")
    ws.package("gsref.backend", base)
    mods = {}
    for name in ("constants", "math_kernels", "preprocess_kernels", "binning_kernels", "render_kernels",
                 "backward_kernels"):
        mods[name] = ws.load_module(f"gsref.backend.{name}", base / f"{name}.py")
    ws.stub("gsref._stream")
    ws.stub("gsref._tuning")
    mods["fused_ssim"] = ws.load_module("gsref.fused_ssim", root / "gswarp" / "fused_ssim.py")
    mods["knn"] = ws.load_module("gsref.knn", root / "gswarp" / "knn.py")
    return mods


def A(x, vec=0):
    return ws.warray(x, vec)


# ------------------------------------------------------------------ scenes
def _unit_quats(n, rng):
    q = rng.normal(size=(n, 4))
    return (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(F32)


def make_scene(name: str):
    """Seeded synthetic scenes (config-2 style distributions, small)."""
    from gswarp_b200 import workloads as wl

    rng = np.random.default_rng({"sh3_64x48": 11, "deg1_bg_50x37": 12, "dense_32x32": 13,
                                 "big_footprints_80x48": 14}[name])
    if name == "sh3_64x48":
        P, W, H, deg, K = 1200, 64, 48, 3, 16
        centres = rng.uniform(-1.0, 1.0, size=(6, 3))
        means = centres[rng.integers(0, 6, P)] + rng.normal(0, 0.35, size=(P, 3))
        log_s = rng.normal(-3.3, 0.5, size=(P, 3))
        eye = [0.3, -0.4, -3.2]
    elif name == "deg1_bg_50x37":
        P, W, H, deg, K = 600, 50, 37, 1, 4
        means = rng.uniform(-1.0, 1.0, size=(P, 3))
        log_s = rng.normal(-3.0, 0.4, size=(P, 3))
        eye = [-0.5, 0.2, -3.0]
    elif name == "dense_32x32":
        P, W, H, deg, K = 2000, 32, 32, 2, 9
        means = rng.normal(0, 0.3, size=(P, 3))
        log_s = rng.normal(-2.8, 0.3, size=(P, 3))
        eye = [0.0, 0.0, -2.5]
    else:  # big_footprints_80x48: AccuTile bands beyond a few tiles, conic_rect rects above 64 tiles
        P, W, H, deg, K = 300, 80, 48, 0, 1
        means = rng.uniform(-0.8, 0.8, size=(P, 3))
        log_s = rng.normal(-2.0, 0.6, size=(P, 3))
        log_s[:, 2] -= 1.5
        eye = [0.1, 0.3, -2.6]
    view = wl.look_at_view(eye, [0.0, 0.0, 0.0], [0.0, -1.0, 0.0], 55.0, W, H)
    sh = np.zeros((P, K, 3), F32)
    sh[:, 0, :] = rng.normal(0, 0.5, size=(P, 3))
    if K > 1:
        sh[:, 1:, :] = rng.normal(0, 0.15, size=(P, K - 1, 3))
    op = 1.0 / (1.0 + np.exp(-rng.normal(0, 1.5, size=(P, 1))))
    op[:5] = [[0.003], [1.0 / 255.0], [0.999], [0.5], [0.02]]  # sub-threshold and boundary opacities
    bg = np.array([0.0, 0.0, 0.0] if name != "deg1_bg_50x37" else [0.2, 0.5, 0.9], F32)
    return dict(
        means=means.astype(F32), scales=np.exp(log_s).astype(F32), rotations=_unit_quats(P, rng),
        opacities=op.astype(F32), sh=sh, degree=np.int32(deg), W=np.int32(W), H=np.int32(H),
        view=view.viewmatrix.numpy().astype(F32), proj=view.projmatrix.numpy().astype(F32),
        campos=view.campos.numpy().astype(F32), tanfovx=np.float64(view.tanfovx),
        tanfovy=np.float64(view.tanfovy), bg=bg,
        grad_color=rng.normal(size=(3, H, W)).astype(F32), grad_depth=rng.normal(size=(1, H, W)).astype(F32),
        grad_alpha=rng.normal(size=(1, H, W)).astype(F32),
        grad_proj_2d=(0.01 * rng.normal(size=(P, 2))).astype(F32),
        grad_conic_2d=(0.01 * rng.normal(size=(P, 3))).astype(F32),
        grad_conic_2d_inv=(0.001 * rng.normal(size=(P, 3))).astype(F32),
    )


# ------------------------------------------------------------------ stages
def preprocess(m, s, mode):
    """preprocess_ops.py:289-581 (scale/rotation path: fused kernel, then SH colour)."""
    pk = m["preprocess_kernels"]
    P, W, H = len(s["means"]), int(s["W"]), int(s["H"])
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    focal_x = W / (2.0 * s["tanfovx"])
    focal_y = H / (2.0 * s["tanfovy"])
    o = dict(cov3d=np.zeros(P * 6, F32), visible=np.zeros(P, np.int32), depths=np.zeros(P, F32),
             radii=np.zeros(P, np.int32), proj_2d=np.zeros((P, 2), F32), conic_2d=np.zeros((P, 3), F32),
             conic_2d_inv=np.zeros((P, 3), F32), points_xy=np.zeros((P, 2), F32),
             tiles_touched=np.zeros(P, np.int32), conic_opacity=np.zeros((P, 4), F32))
    ws.launch(pk._fused_project_cov3d_cov2d_preprocess_sr_warp_kernel, P, [
        A(s["means"], 3), A(s["scales"], 3), A(s["rotations"], 4), F32(1.0), A(s["opacities"].reshape(-1)),
        A(s["view"].reshape(-1)), A(s["proj"].reshape(-1)), F32(s["tanfovx"]), F32(s["tanfovy"]),
        F32(focal_x), F32(focal_y), W, H, gx, gy, mode,
        A(o["cov3d"]), A(o["visible"]), A(o["depths"]), A(o["radii"]), A(o["proj_2d"], 2), A(o["conic_2d"], 3),
        A(o["conic_2d_inv"], 3), A(o["points_xy"], 2), A(o["tiles_touched"]), A(o["conic_opacity"], 4)])
    # _compute_rgb_from_sh_warp (preprocess_ops.py:239-286)
    K = s["sh"].shape[1]
    o["rgb"] = np.zeros((P, 3), F32)
    o["clamped"] = np.zeros(P * 3, np.int32)
    ws.launch(pk._forward_rgb_from_sh_v3_warp_kernel, P, [
        A(s["means"], 3), A(s["campos"].reshape(-1)), A(s["sh"].reshape(-1, 3), 3), int(s["degree"]), K,
        A(o["rgb"], 3), A(o["clamped"])])
    o["clamped"] = o["clamped"].reshape(P, 3)
    return o


def binning(m, pre, W, H, mode):
    """binning_ops.py:84-431, sort mode 'warp_depth_stable_tile' (the default)."""
    bk = m["binning_kernels"]
    P = len(pre["radii"])
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    tiles = gx * gy
    tiles_touched = pre["tiles_touched"].copy()
    if mode == 2:  # :105-137
        masks = np.zeros(P, np.int64)
        ws.launch(bk._recount_covered_tiles_warp_kernel, P, [
            A(pre["points_xy"], 2), A(pre["radii"]), A(pre["conic_opacity"], 4), A(pre["conic_2d_inv"], 3),
            gx, gy, mode, A(tiles_touched), A(masks)])
    else:
        masks = np.zeros(1, np.int64)
    # depth sort with the packed payload (:141-205)
    point_bits = (P - 1).bit_length()
    assert point_bits + tiles.bit_length() <= 31
    keys = np.zeros(P, np.int32)
    payload = np.zeros(P, np.int32)
    ws.launch(bk._prepare_depth_sort_payload_warp_kernel, P, [
        A(pre["depths"].view(np.int32)), A(tiles_touched), point_bits, 1, A(keys), A(payload)])
    order = np.argsort(keys, kind="stable")  # Warp radix_sort_pairs: stable by key
    payload = payload[order]
    ids = np.zeros(P, np.int32)
    sorted_tt = np.zeros(P, np.int32)
    ws.launch(bk._unpack_depth_sort_payload_warp_kernel, P, [
        A(payload), point_bits, (1 << point_bits) - 1, A(ids), A(sorted_tt)])
    offsets = np.cumsum(sorted_tt).astype(np.int32)  # _inclusive_scan_i32
    R = int(offsets[-1]) if P else 0
    tile_ids = np.zeros(max(R, 1), np.int32)
    point_list = np.zeros(max(R, 1), np.int32)
    ws.launch(bk._duplicate_with_keys_from_order_warp_kernel, P, [
        A(pre["points_xy"], 2), A(pre["radii"]), A(pre["conic_opacity"], 4), A(pre["conic_2d_inv"], 3),
        A(ids), A(offsets), gx, gy, mode, A(masks), A(tile_ids), A(point_list)])
    tile_ids, point_list = tile_ids[:R], point_list[:R]
    order = np.argsort(tile_ids, kind="stable")  # stable i32 radix sort by tile id
    tile_ids, point_list = tile_ids[order], point_list[order]
    ranges = np.zeros((tiles + 1) * 2, np.int32)
    ws.launch(bk._identify_tile_ranges_warp_kernel, R, [A(tile_ids), A(ranges), R])
    return dict(tiles_touched=tiles_touched, point_list=point_list,
                ranges=ranges.reshape(-1, 2)[:tiles].copy(), depth_order=ids, offsets=offsets)


def render_fwd(m, pre, b, s, compute_depth):
    """render_ops.py:16-93 (tiled 256-thread blocks)."""
    W, H = int(s["W"]), int(s["H"])
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    nt = gx * gy
    color = np.zeros(3 * H * W, F32)
    depth = np.zeros(H * W, F32)
    alpha = np.zeros(H * W, F32)
    nc = np.zeros(H * W, np.int32)
    ws.launch(m["render_kernels"]._render_tiles_tiled256_warp_kernel, nt * 256, [
        A(b["ranges"].reshape(-1)), A(b["point_list"]), A(pre["points_xy"], 2), A(pre["rgb"].reshape(-1)),
        A(pre["depths"]), A(pre["conic_opacity"], 4), A(s["bg"]), W, H, gx, nt, int(compute_depth),
        A(color), A(depth), A(alpha), A(nc)], block_dim=256)
    return dict(color=color.reshape(3, H, W), depth=depth.reshape(1, H, W), alpha=alpha.reshape(1, H, W),
                n_contrib=nc)


def render_bwd(m, pre, b, f, s, compute_depth):
    """backward_ops.py:183-290 (warp32 kernel, 32-thread blocks); the
    gradient sums are float64 (see the module docstring)."""
    W, H = int(s["W"]), int(s["H"])
    P = len(pre["radii"])
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    nt = gx * gy
    g_xy = np.zeros((P, 2), np.float64)
    g_d = np.zeros(P, np.float64)
    g_co = np.zeros((P, 4), np.float64)
    g_f = np.zeros((P, 3), np.float64)
    ws.launch(m["backward_kernels"]._backward_render_tiles_warp32_kernel, nt * 256, [
        A(b["ranges"].reshape(-1)), A(b["point_list"]), A(pre["points_xy"], 2), A(pre["rgb"].reshape(-1)),
        A(pre["depths"]), A(pre["conic_opacity"], 4), A(s["bg"]), A(f["alpha"].reshape(-1)), A(f["n_contrib"]),
        A(s["grad_color"].reshape(-1)), A(s["grad_depth"].reshape(-1)), A(s["grad_alpha"].reshape(-1)),
        W, H, gx, nt, int(compute_depth), A(g_xy, 2), A(g_d), A(g_co, 4), A(g_f, 3)], block_dim=32)
    return dict(grad_xy=g_xy, grad_depth=g_d, grad_conic_opacity=g_co, grad_rgb=g_f)


def preprocess_bwd(m, pre, s, rg):
    """backward_ops.py:525-680: SH backward (:51-149; the (K,P,3) layout for
    degree > 1), then the fused preprocess backward.  ``rg`` are the render
    gradients as float32 (the reference's own buffers are float32)."""
    bk = m["backward_kernels"]
    P, W, H = len(s["means"]), int(s["W"]), int(s["H"])
    K = s["sh"].shape[1]
    deg = int(s["degree"])
    grad_mean_sh = np.zeros((P, 3), F32)
    if deg <= 1:
        grad_sh = np.zeros(P * K * 3, F32)
        ws.launch(bk._backward_rgb_from_sh_warp_kernel, P, [
            A(s["means"], 3), A(s["campos"].reshape(-1)), A(s["sh"].reshape(-1)), deg, K,
            A(pre["clamped"].reshape(-1)), A(rg["grad_rgb"].reshape(-1)), A(grad_mean_sh, 3), A(grad_sh)])
        grad_sh = grad_sh.reshape(P, K, 3)
    else:
        soa = np.ascontiguousarray(s["sh"].transpose(1, 0, 2)).reshape(-1, 3)
        g_soa = np.zeros((K * P, 3), F32)
        ws.launch(bk._backward_rgb_from_sh_v3_warp_kernel, P, [
            A(s["means"], 3), A(s["campos"].reshape(-1)), A(soa, 3), deg, K, P, A(rg["grad_rgb"], 3),
            A(pre["clamped"].reshape(-1)), A(grad_mean_sh, 3), A(g_soa, 3)])
        grad_sh = np.ascontiguousarray(g_soa.reshape(K, P, 3).transpose(1, 0, 2))
    focal_x = W / (2.0 * s["tanfovx"])
    focal_y = H / (2.0 * s["tanfovy"])
    out = dict(grad_means3d=np.zeros((P, 3), F32), grad_means2d=np.zeros((P, 3), F32),
               grad_scales=np.zeros((P, 3), F32), grad_rotations=np.zeros((P, 4), F32))
    ws.launch(bk._fused_backward_preprocess_accumulate_warp_kernel, P, [
        A(s["means"], 3), A(pre["radii"]), A(s["proj"].reshape(-1)), A(s["view"].reshape(-1)),
        A(rg["grad_xy"], 2), A(s["grad_proj_2d"], 2), A(rg["grad_depth"]), A(pre["cov3d"]),
        F32(s["tanfovx"]), F32(s["tanfovy"]), F32(focal_x), F32(focal_y), F32(0.0),
        A(rg["grad_conic_opacity"], 4), A(s["grad_conic_2d"].reshape(-1)), A(s["grad_conic_2d_inv"].reshape(-1)),
        A(s["scales"], 3), A(s["rotations"], 4), F32(1.0), A(grad_mean_sh, 3), 1, A(rg["grad_xy"], 2),
        A(out["grad_means3d"], 3), A(out["grad_means2d"], 3), A(out["grad_scales"], 3),
        A(out["grad_rotations"], 4)])
    out["grad_sh"] = grad_sh
    out["grad_opacity"] = rg["grad_conic_opacity"][:, 3].copy()
    return out


def scene_golden(m, name: str) -> dict:
    s = make_scene(name)
    W, H = int(s["W"]), int(s["H"])
    res = {f"in_{k}": v for k, v in s.items()}
    t0 = time.time()
    pre = {}
    for mode in (1, 0, 2):
        p = preprocess(m, s, mode)
        b = binning(m, p, W, H, mode)
        for k in ("radii", "depths", "proj_2d", "conic_2d", "conic_2d_inv", "tiles_touched", "conic_opacity",
                  "rgb", "clamped", "cov3d"):
            res[f"m{mode}_pre_{k}"] = p[k]
        res[f"m{mode}_bin_tiles_touched"] = b["tiles_touched"]
        res[f"m{mode}_bin_point_list"] = b["point_list"]
        res[f"m{mode}_bin_ranges"] = b["ranges"]
        if mode == 1:
            pre, bins = p, b
    print(f"  {name}: preprocess+binning x3 {time.time() - t0:.1f}s, R={len(bins['point_list'])}", flush=True)
    for cd in (1, 0):
        t0 = time.time()
        f = render_fwd(m, pre, bins, s, cd)
        for k, v in f.items():
            res[f"fwd{cd}_{k}"] = v
        print(f"  {name}: render fwd (depth={cd}) {time.time() - t0:.1f}s", flush=True)
        if cd == 1:
            fwd = f
    t0 = time.time()
    rb = render_bwd(m, pre, bins, fwd, s, 1)
    for k, v in rb.items():
        res[f"bwd_{k}"] = v
    print(f"  {name}: render bwd {time.time() - t0:.1f}s", flush=True)
    rg = {k: v.astype(F32) for k, v in rb.items()}
    pb = preprocess_bwd(m, pre, s, rg)
    for k, v in pb.items():
        res[f"pbwd_{k}"] = v
    return res


# --------------------------------------------------------------------- SSIM
def ssim_golden(m) -> dict:
    """FusedSSIMMap training plan (fused_ssim.py:127-288): H pass, V pass
    (tiled for 'same'), mean of the map, backward H and V passes with
    upstream 1."""
    fs = m["fused_ssim"]
    rng = np.random.default_rng(21)
    B, C, H, W = 2, 3, 37, 53
    x = rng.uniform(0, 1, size=(B, C, H, W)).astype(F32)
    y = np.clip(x + rng.normal(0, 0.05, size=x.shape), 0, 1).astype(F32)
    res = dict(in_img1=x, in_img2=y)
    N = x.size
    C1, C2 = 0.01 ** 2, 0.03 ** 2
    for valid in (0, 1):
        hbuf = np.zeros(4 * N, F32)
        hs = [hbuf[i * N:(i + 1) * N] for i in range(4)]
        h3 = [h.reshape(B * C, H, W) for h in hs]
        dm = np.zeros(3 * N, F32)
        dms = [dm[i * N:(i + 1) * N] for i in range(3)]
        ws.launch(fs._fwd_h, N, [A(x.reshape(-1)), A(y.reshape(-1)), *map(A, hs), W])
        if valid:
            Hv, Wv = H - 10, W - 10
            ssim = np.zeros(B * C * Hv * Wv, F32)
            ws.launch(fs._fwd_v_train_valid, ssim.size, [*map(A, hs), A(ssim), *map(A, dms), H, W, Hv, Wv,
                                                         F32(C1), F32(C2)])
            smap = ssim.reshape(B, C, Hv, Wv)
        else:
            tx, ty = (W + 31) // 32, (H + 7) // 8
            ssim = np.zeros(N, F32)
            ws.launch(fs._fwd_v_train_tiled, B * C * tx * ty * 256, [
                *map(A, h3), A(ssim), *map(A, dms), H, W, tx, ty, F32(C1), F32(C2)], block_dim=256)
            smap = ssim.reshape(B, C, H, W)
        nvalid = smap.size
        up = np.ones(1, F32)
        ts = [hbuf[i * N:(i + 1) * N] for i in range(3)]  # the plan reuses the H buffers
        grad = np.zeros(N, F32)
        if valid:
            ws.launch(fs._bwd_h_scalar_valid, N, [*map(A, dms), *map(A, ts), H, W, F32(1.0 / float(nvalid)), A(up)])
            ws.launch(fs._bwd_v, N, [A(x.reshape(-1)), A(y.reshape(-1)), *map(A, ts), A(grad), H, W])
        else:
            ws.launch(fs._bwd_h_scalar, N, [*map(A, dms), *map(A, ts), W, F32(1.0 / float(N)), A(up)])
            ws.launch(fs._bwd_v_tiled, B * C * tx * ty * 256, [
                A(x.reshape(-1)), A(y.reshape(-1)), *[A(t.reshape(B * C, H, W)) for t in ts], A(grad), H, W, tx, ty],
                block_dim=256)
        tag = "valid" if valid else "same"
        res[f"{tag}_map"] = smap
        res[f"{tag}_dm"] = dm.reshape(3, B, C, H, W)
        res[f"{tag}_grad"] = grad.reshape(B, C, H, W)
    return res


# ---------------------------------------------------------------------- KNN
def knn_golden(m) -> dict:
    """_distCUDA2_impl (knn.py:264-401)."""
    kn = m["knn"]
    rng = np.random.default_rng(31)
    P = 1500
    centres = rng.uniform(-20, 20, size=(12, 3))
    sig = rng.uniform(0.05, 1.5, size=(12, 3))
    c = rng.integers(0, 12, P)
    pts = centres[c] + rng.normal(size=(P, 3)) * sig[c]
    pts[:75] = rng.uniform(-20, 20, size=(75, 3))  # 5% outliers
    pts[100:110] = pts[90]  # exact duplicates (zero distances, ties)
    pts = pts.astype(F32)
    mn, mx = pts.min(axis=0).astype(np.float64), pts.max(axis=0).astype(np.float64)
    eps = 1e-7
    for i in range(3):
        if mx[i] - mn[i] < eps:
            mx[i] = mn[i] + eps
    codes = np.zeros(P, np.uint32)
    ws.launch(kn._coord2morton_kernel, P, [A(pts), *[F32(v) for v in mn], *[F32(v) for v in mx], A(codes)])
    order = np.argsort(codes.view(np.int32), kind="stable").astype(np.int32)  # radix_sort_pairs (int32 keys)
    sx, sy, sz = (np.zeros(P, F32) for _ in range(3))
    ws.launch(kn._gather_sorted_soa_kernel, P, [A(pts), A(order), A(sx), A(sy), A(sz)])
    nb = (P + 1023) // 1024
    bmin = [np.full(nb, np.inf, F32) for _ in range(3)]
    bmax = [np.full(nb, -np.inf, F32) for _ in range(3)]
    ws.launch(kn._box_min_max_kernel, P, [A(sx), A(sy), A(sz), *map(A, bmin), *map(A, bmax), P])
    d = np.zeros(P, F32)
    ws.launch(kn._box_mean_dist_kernel, P, [A(sx), A(sy), A(sz), A(order), *map(A, bmin), *map(A, bmax), nb, P,
                                            A(d)])
    return dict(in_points=pts, codes=codes, order=order, dists=d)


def main(argv):
    if not argv:
        print(__doc__)
        return 2
    root = Path(argv[0]).resolve()
    names = argv[1:] or ["sh3_64x48", "deg1_bg_50x37", "dense_32x32", "big_footprints_80x48", "ssim", "knn"]
    m = load_reference(root)
    for name in names:
        t0 = time.time()
        if name == "ssim":
            res = ssim_golden(m)
        elif name == "knn":
            res = knn_golden(m)
        else:
            res = scene_golden(m, name)
        res["source"] = np.array(f"gswarp kernel code run by tests/golden/make_kernel_golden.py ({name})")
        dst = HERE / f"kernels_{name}.npz"
        np.savez_compressed(dst, **res)
        print(f"{name}: {time.time() - t0:.1f}s -> {dst.name} ({dst.stat().st_size // 1024} KiB)", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
