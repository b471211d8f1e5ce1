"""Seeded synthetic scenes with the shapes and distributions of the
benchmark configurations (there is no dataset on the box).

Camera matrices follow the 3DGS convention the kernels read: ``viewmatrix``
is the transposed world-to-camera matrix and ``projmatrix`` the transposed
full projection, both flattened column-major by the kernels (flat[c*4+r]).
The camera looks down +z (x right, y down).  All generation happens on the
CPU with ``torch.Generator`` so every box produces the same inputs.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class View:
    width: int
    height: int
    tanfovx: float
    tanfovy: float
    viewmatrix: torch.Tensor  # (4,4) transposed world->view
    projmatrix: torch.Tensor  # (4,4) transposed full projection
    campos: torch.Tensor      # (3,)

    def to(self, device):
        return View(self.width, self.height, self.tanfovx, self.tanfovy, self.viewmatrix.to(device),
                    self.projmatrix.to(device), self.campos.to(device))


def look_at_view(eye, target, up, fovx_deg: float, width: int, height: int, znear=0.01, zfar=100.0) -> View:
    eye = torch.as_tensor(eye, dtype=torch.float64)
    target = torch.as_tensor(target, dtype=torch.float64)
    up = torch.as_tensor(up, dtype=torch.float64)
    f = target - eye
    f = f / f.norm()
    r = torch.linalg.cross(f, up)
    if r.norm() < 1e-9:
        r = torch.linalg.cross(f, torch.tensor([1.0, 0.0, 0.0], dtype=torch.float64))
    r = r / r.norm()
    d = torch.linalg.cross(f, r)
    Rm = torch.stack([r, d, f])               # rows: camera axes
    t = -Rm @ eye
    w2v = torch.eye(4, dtype=torch.float64)
    w2v[:3, :3] = Rm
    w2v[:3, 3] = t
    tanfovx = math.tan(math.radians(fovx_deg) / 2.0)
    tanfovy = tanfovx * height / width
    top, right = tanfovy * znear, tanfovx * znear
    Pm = torch.zeros(4, 4, dtype=torch.float64)
    Pm[0, 0] = 2.0 * znear / (2 * right)
    Pm[1, 1] = 2.0 * znear / (2 * top)
    Pm[3, 2] = 1.0
    Pm[2, 2] = zfar / (zfar - znear)
    Pm[2, 3] = -(zfar * znear) / (zfar - znear)
    full = Pm @ w2v
    return View(width, height, tanfovx, tanfovy, w2v.T.contiguous().float(), full.T.contiguous().float(),
                eye.float())


@dataclass
class Scene:
    means: torch.Tensor
    scales: torch.Tensor
    rotations: torch.Tensor
    opacities: torch.Tensor
    sh: torch.Tensor          # (N, K, 3)
    sh_degree: int

    def to(self, device):
        return Scene(self.means.to(device), self.scales.to(device), self.rotations.to(device),
                     self.opacities.to(device), self.sh.to(device), self.sh_degree)

    @property
    def n(self) -> int:
        return self.means.shape[0]


def _unit_quats(n, g):
    q = torch.randn(n, 4, generator=g)
    return q / q.norm(dim=1, keepdim=True)


def config1_scene(seed: int = 0, n: int = 10_000):
    """10K Gaussians, means U[-1,1]^3, log-scales N(-3.5,0.4), normalised
    quaternions, opacity sigmoid(N(0,1)), SH degree 0 DC N(0,0.3) (N,1,3);
    256x256 pinhole at distance 3 looking at the origin, FoV 60 deg."""
    g = torch.Generator().manual_seed(seed)
    means = torch.rand(n, 3, generator=g) * 2.0 - 1.0
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.4 - 3.5)
    rots = _unit_quats(n, g)
    opac = torch.sigmoid(torch.randn(n, 1, generator=g))
    sh = torch.randn(n, 1, 3, generator=g) * 0.3
    view = look_at_view([0.0, 0.0, -3.0], [0.0, 0.0, 0.0], [0.0, -1.0, 0.0], 60.0, 256, 256)
    return Scene(means, scales, rots, opac, sh, 0), view


def _cluster_means(n, clusters, g, box=5.0, sigma=0.8):
    centres = (torch.rand(clusters, 3, generator=g) * 2.0 - 1.0) * box
    assign = torch.randint(0, clusters, (n,), generator=g)
    return centres[assign] + torch.randn(n, 3, generator=g) * sigma


def config2_scene(seed: int = 0, n: int = 1_000_000):
    """Mixture of 64 isotropic clusters (centres U[-5,5]^3, sigma 0.8),
    log-scales N(-4.5,0.6), random unit quaternions, opacity
    sigmoid(N(0,1.5)), SH degree 3 (N,16,3) with DC N(0,0.5) and higher bands
    N(0,0.05)."""
    g = torch.Generator().manual_seed(seed)
    means = _cluster_means(n, 64, g)
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.6 - 4.5)
    rots = _unit_quats(n, g)
    opac = torch.sigmoid(torch.randn(n, 1, generator=g) * 1.5)
    sh = torch.randn(n, 16, 3, generator=g) * 0.05
    sh[:, 0, :] = torch.randn(n, 3, generator=g) * 0.5
    return Scene(means, scales, rots, opac, sh, 3)


def config2_view(seed: int = 0, width: int = 1920, height: int = 1080) -> View:
    """Camera at radius 12 on a seeded random direction looking at the origin, FoVx 50 deg."""
    g = torch.Generator().manual_seed(seed + 7919)
    d = torch.randn(3, generator=g, dtype=torch.float64)
    d = d / d.norm()
    return look_at_view((12.0 * d).tolist(), [0.0, 0.0, 0.0], [0.0, 0.0, 1.0], 50.0, width, height)


def ring_views(count: int = 64, seed: int = 0, width: int = 1920, height: int = 1080) -> list[View]:
    """Cameras on a ring of radius 12 at random elevations in [-20, 30] deg."""
    g = torch.Generator().manual_seed(seed + 104729)
    elev = torch.rand(count, generator=g, dtype=torch.float64) * 50.0 - 20.0
    views = []
    for i in range(count):
        az = 2.0 * math.pi * i / count
        el = math.radians(float(elev[i]))
        eye = [12.0 * math.cos(el) * math.cos(az), 12.0 * math.cos(el) * math.sin(az), 12.0 * math.sin(el)]
        views.append(look_at_view(eye, [0.0, 0.0, 0.0], [0.0, 0.0, 1.0], 50.0, width, height))
    return views


def target_image(seed: int, height: int = 1080, width: int = 1920) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 31337)
    return torch.rand(3, height, width, generator=g)


def config3_images(seed: int = 0, shape=(4, 3, 1080, 1920)):
    """SSIM pair: U[0,1] images and clamp(img + N(0,0.05), 0, 1)."""
    g = torch.Generator().manual_seed(seed)
    img = torch.rand(*shape, generator=g)
    tgt = (img + torch.randn(*shape, generator=g) * 0.05).clamp(0.0, 1.0)
    return img, tgt


def config4_points(seed: int = 0, n: int = 2_000_000):
    """256 anisotropic clusters (centres U[-20,20]^3, per-axis sigma
    U[0.05,1.5]) plus 5% uniform outliers in the same box."""
    g = torch.Generator().manual_seed(seed)
    n_out = int(round(n * 0.05))
    n_in = n - n_out
    centres = (torch.rand(256, 3, generator=g) * 2.0 - 1.0) * 20.0
    sig = torch.rand(256, 3, generator=g) * 1.45 + 0.05
    assign = torch.randint(0, 256, (n_in,), generator=g)
    pts = centres[assign] + torch.randn(n_in, 3, generator=g) * sig[assign]
    outl = (torch.rand(n_out, 3, generator=g) * 2.0 - 1.0) * 20.0
    allp = torch.cat([pts, outl])
    perm = torch.randperm(n, generator=g)
    return allp[perm].contiguous()
