"""Seeded synthetic workloads of the benchmark configurations.

The reference publishes no datasets or benchmark scenes for this path, so the
inputs are synthetic, drawn on the CPU in fp32 from
``torch.Generator().manual_seed(20261201 + config_index)``:

  0  imagegs_small : Image-GS fit step, 256x256 RGB, 4,096 Gaussians
  1  imagegs_large : Image-GS fit step, 2048x2048 RGB, 100,000 Gaussians
  2  hexels2d      : 2D image hexels, 1024x1024 RGB, 50,000 hexagons

Image-GS: means2d ~ U[0,1)^2, scales2d = exp(N(ln s0, 0.5)) pixels
(s0 = 2 at 256^2; scaled with the image, s0 = 16 at 2048^2), rotation ~
U[0, 2pi), colours ~ U[0,1], target image ~ U[0,1]; top-K=10 normalised
weighted sum, 16x16 tiles, loss = mean((img - target)^2).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict

import torch

SEED_BASE = 20261201


@dataclass
class ImageGSWorkload:
    name: str
    height: int
    width: int
    means2d: torch.Tensor
    scales2d: torch.Tensor
    rotation: torch.Tensor
    colors: torch.Tensor
    target: torch.Tensor
    extra: Dict[str, float] = field(default_factory=dict)

    @property
    def num_points(self) -> int:
        return self.means2d.shape[0]

    @property
    def tile_bounds(self):
        return ((self.width + 15) // 16, (self.height + 15) // 16, 1)

    def to(self, device) -> "ImageGSWorkload":
        kw = {k: getattr(self, k).to(device) for k in
              ("means2d", "scales2d", "rotation", "colors", "target")}
        return ImageGSWorkload(self.name, self.height, self.width, extra=dict(self.extra), **kw)


def imagegs(config_index: int, height: int, width: int, num_points: int, scale_px: float,
            name: str) -> ImageGSWorkload:
    g = torch.Generator().manual_seed(SEED_BASE + config_index)
    means2d = torch.rand((num_points, 2), generator=g, dtype=torch.float32)
    scales2d = torch.exp(math.log(scale_px) + 0.5 * torch.randn((num_points, 2), generator=g))
    rotation = 2 * math.pi * torch.rand((num_points, 1), generator=g, dtype=torch.float32)
    colors = torch.rand((num_points, 3), generator=g, dtype=torch.float32)
    target = torch.rand((height, width, 3), generator=g, dtype=torch.float32)
    return ImageGSWorkload(name, height, width, means2d, scales2d.float(), rotation, colors,
                           target, {"scale_px": scale_px})


def imagegs_small() -> ImageGSWorkload:
    return imagegs(0, 256, 256, 4096, 2.0, "imagegs_small_256x256_n4096")


def imagegs_large() -> ImageGSWorkload:
    return imagegs(1, 2048, 2048, 100_000, 2.0 * 2048 / 256, "imagegs_large_2048x2048_n100000")


def imagegs_tiny(seed: int = 7, height: int = 48, width: int = 72, num_points: int = 96,
                 scale_px: float = 3.0) -> ImageGSWorkload:
    """Small ragged case for parity tests (image not a multiple of 16)."""
    return imagegs(1000 + seed, height, width, num_points, scale_px,
                   f"imagegs_tiny_{height}x{width}_n{num_points}")


@dataclass
class HexelsWorkload:
    """2D image hexels: pixel-space centres, scale/rotation geometry and the
    binning radius the caller uses (the reference's hexel kernels take their
    binning from the caller)."""

    name: str
    height: int
    width: int
    xys: torch.Tensor        # (N,2) pixel centres
    scales: torch.Tensor     # (N,2)
    rotation: torch.Tensor   # (N,1)
    colors: torch.Tensor     # (N,3)
    radii: torch.Tensor      # (N,) int32 binning radius in pixels
    target: torch.Tensor
    softness: float = 10.0
    aa_kernel_size: float = 0.0
    extra: Dict[str, torch.Tensor] = field(default_factory=dict)

    @property
    def num_points(self) -> int:
        return self.xys.shape[0]

    @property
    def tile_bounds(self):
        return ((self.width + 15) // 16, (self.height + 15) // 16, 1)


def hexels(config_index: int, height: int, width: int, num_points: int, radius_px: float,
           softness: float, name: str) -> HexelsWorkload:
    """Centres ~ U[0,W) x U[0,H), circumradius R = exp(N(ln r0, 0.4)) pixels,
    scales = (R sqrt(3)/2, R sqrt(3)/2) (the SDF's circumradius along u is
    (2/sqrt(3)) s_x and its apothem along v is s_y), rotation ~ U[0, pi/3),
    colours ~ U[0,1].  The opacity ~ sigmoid(N(0,1)) draw of the configuration
    is made (to keep the random stream) but is not an input of these kernels.
    Binning radius: ceil(R (1 + ln(254) / softness)) + 1 pixels."""
    g = torch.Generator().manual_seed(SEED_BASE + config_index)
    xys = torch.rand((num_points, 2), generator=g) * torch.tensor([float(width), float(height)])
    R = torch.exp(math.log(radius_px) + 0.4 * torch.randn((num_points,), generator=g))
    s = R * (math.sqrt(3.0) / 2.0)
    scales = torch.stack([s, s], 1).float()
    rotation = (math.pi / 3.0) * torch.rand((num_points, 1), generator=g)
    colors = torch.rand((num_points, 3), generator=g)
    opacity = torch.sigmoid(torch.randn((num_points,), generator=g))
    target = torch.rand((height, width, 3), generator=g)
    radii = (torch.ceil(R * (1.0 + math.log(254.0) / softness)) + 1).to(torch.int32)
    return HexelsWorkload(name, height, width, xys.float(), scales, rotation.float(), colors,
                          radii, target, softness, 0.0, {"opacity_unused": opacity})


@dataclass
class Camera:
    """A pinhole camera in the 3DGS convention: viewmatrix = world->view
    transposed, projmatrix = (projection @ world->view) transposed, both
    stored row-major as the kernels read them."""

    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    campos: torch.Tensor
    width: int
    height: int
    tan_fovx: float
    tan_fovy: float

    def to(self, device) -> "Camera":
        return Camera(self.viewmatrix.to(device), self.projmatrix.to(device),
                      self.campos.to(device), self.width, self.height, self.tan_fovx,
                      self.tan_fovy)


def look_at_camera(center, width: int, height: int, fx: float, fy: float,
                   znear: float = 0.01, zfar: float = 100.0) -> Camera:
    """Camera at `center` looking at the origin with +y up (view space: x
    right, y down, z forward)."""
    C = torch.tensor(center, dtype=torch.float64)
    z = -C / C.norm()
    y = torch.tensor([0.0, -1.0, 0.0], dtype=torch.float64)
    y = y - (y @ z) * z
    y = y / y.norm()
    x = torch.linalg.cross(y, z)
    R = torch.stack([x, y, z])  # rows: view axes in world coordinates
    w2v = torch.eye(4, dtype=torch.float64)
    w2v[:3, :3] = R
    w2v[:3, 3] = -R @ C
    tan_x = width / (2.0 * fx)
    tan_y = height / (2.0 * fy)
    top, right = tan_y * znear, tan_x * znear
    P = torch.zeros((4, 4), dtype=torch.float64)
    P[0, 0] = 2.0 * znear / (2 * right)
    P[1, 1] = 2.0 * znear / (2 * top)
    P[3, 2] = 1.0
    P[2, 2] = zfar / (zfar - znear)
    P[2, 3] = -(zfar * znear) / (zfar - znear)
    view = w2v.T.contiguous().float()
    proj = (P @ w2v).T.contiguous().float()
    return Camera(view, proj, C.float(), width, height, tan_x, tan_y)


@dataclass
class Hexels3DWorkload:
    """3D hexel surfels: means (P,3), tangent scales (P,2), WXYZ rotations
    (P,4), opacities (P,), colours (P,3), linear colour gradients (P,2,3),
    linear view gradients (P,3,3)."""

    name: str
    means3d: torch.Tensor
    scales: torch.Tensor
    rotations: torch.Tensor
    opacities: torch.Tensor
    colors: torch.Tensor
    color_grads: torch.Tensor
    view_grads: torch.Tensor
    background: torch.Tensor
    cameras: list
    softness: float = 10.0

    @property
    def num_points(self) -> int:
        return self.means3d.shape[0]

    def to(self, device) -> "Hexels3DWorkload":
        f = lambda t: t.to(device)  # noqa: E731
        return Hexels3DWorkload(self.name, f(self.means3d), f(self.scales), f(self.rotations),
                                f(self.opacities), f(self.colors), f(self.color_grads),
                                f(self.view_grads), f(self.background),
                                [c.to(device) for c in self.cameras], self.softness)


def hexels3d(config_index: int, num_points: int, width: int, height: int, focal: float,
             num_views: int, scale: float, name: str) -> Hexels3DWorkload:
    """means ~ U[-1,1]^3, scales = exp(N(ln s0, 0.5)), rotations = normalised
    N(0, I4) (WXYZ), opacities = sigmoid(N(0,1)), colours ~ U[0,1], colour and
    view gradients ~ N(0, 0.1) (the reference's linear colour and linear view
    models stand in for the configuration's spherical-harmonics colours, which
    the reference does not implement), background 0, softness 10.  Cameras on
    a radius-3 orbit in the xz-plane (azimuth 2 pi k / views) looking at the
    origin; view 0 is at (0, 0, 3)."""
    g = torch.Generator().manual_seed(SEED_BASE + config_index)
    P = num_points
    means = torch.rand((P, 3), generator=g) * 2 - 1
    scales = torch.exp(math.log(scale) + 0.5 * torch.randn((P, 2), generator=g))
    q = torch.randn((P, 4), generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    opacities = torch.sigmoid(torch.randn((P,), generator=g))
    colors = torch.rand((P, 3), generator=g)
    color_grads = 0.1 * torch.randn((P, 2, 3), generator=g)
    view_grads = 0.1 * torch.randn((P, 3, 3), generator=g)
    cams = []
    for k in range(num_views):
        th = 2 * math.pi * k / num_views
        cams.append(look_at_camera((3 * math.sin(th), 0.0, 3 * math.cos(th)), width, height,
                                   focal, focal))
    return Hexels3DWorkload(name, means.float(), scales.float(), q.float(), opacities.float(),
                            colors.float(), color_grads.float(), view_grads.float(),
                            torch.zeros(3), cams)


def hexels3d_single() -> Hexels3DWorkload:
    return hexels3d(3, 1_000_000, 1920, 1080, 1100.0, 1, 0.01, "hexels3d_1920x1080_p1000000")


def hexels3d_multiview(num_views: int = 64) -> Hexels3DWorkload:
    return hexels3d(4, 1_000_000, 1920, 1080, 1100.0, num_views, 0.01,
                    f"hexels3d_{num_views}views_1920x1080_p1000000")


def hexels3d_tiny(seed: int = 1, num_points: int = 1500, width: int = 88, height: int = 72,
                  num_views: int = 2, scale: float = 0.06) -> Hexels3DWorkload:
    return hexels3d(3000 + seed, num_points, width, height, width * 1.2, num_views, scale,
                    f"hexels3d_tiny_{width}x{height}_p{num_points}")


def hexels2d() -> HexelsWorkload:
    return hexels(2, 1024, 1024, 50_000, 4.0, 10.0, "hexels2d_1024x1024_n50000")


def hexels2d_tiny(seed: int = 3, height: int = 40, width: int = 56,
                  num_points: int = 60) -> HexelsWorkload:
    return hexels(2000 + seed, height, width, num_points, 4.0, 10.0,
                  f"hexels2d_tiny_{height}x{width}_n{num_points}")
