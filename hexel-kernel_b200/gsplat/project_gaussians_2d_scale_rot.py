"""2D Gaussian projection — same API as the reference's
gsplat/project_gaussians_2d_scale_rot.py:12-113."""

from typing import Tuple

import torch
from torch import Tensor
from torch.autograd import Function

import gsplat.cuda as _C


def project_gaussians_2d_scale_rot(
    means2d: Tensor,
    scales2d: Tensor,
    rotation: Tensor,
    img_height: int,
    img_width: int,
    tile_bounds: Tuple[int, int, int],
) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """Pixel centres, int radii, conics and tile counts of 2D Gaussians given
    normalised means (N,2) in [0,1], pixel scales (N,2) and rotations (N,1)."""
    return _ProjectGaussians2dScaleRot.apply(
        means2d.contiguous(),
        scales2d.contiguous(),
        rotation.contiguous(),
        img_height,
        img_width,
        tile_bounds,
    )


class _ProjectGaussians2dScaleRot(Function):
    """Project 2D scale/rotation Gaussians to pixel space."""

    @staticmethod
    def forward(ctx, means2d, scales2d, rotation, img_height, img_width, tile_bounds):
        num_points = means2d.shape[-2]
        if num_points < 1 or means2d.shape[-1] != 2:
            raise ValueError(f"Invalid shape for means2d: {means2d.shape}")
        xys, radii, conics, num_tiles_hit = _C.project_gaussians_2d_scale_rot_forward(
            num_points, means2d, scales2d, rotation, img_height, img_width, tile_bounds
        )
        ctx.img_height = img_height
        ctx.img_width = img_width
        ctx.num_points = num_points
        ctx.save_for_backward(means2d, scales2d, rotation, radii, conics)
        ctx.mark_non_differentiable(radii, num_tiles_hit)
        return xys, radii, conics, num_tiles_hit

    @staticmethod
    def backward(ctx, v_xys, v_radii, v_conics, v_num_tiles_hit):
        means2d, scales2d, rotation, radii, conics = ctx.saved_tensors
        if v_xys is None:
            v_xys = torch.zeros_like(means2d)
        if v_conics is None:
            v_conics = torch.zeros_like(conics)
        _, v_mean2d, v_scale, v_rot = _C.project_gaussians_2d_scale_rot_backward(
            ctx.num_points,
            means2d,
            scales2d,
            rotation,
            ctx.img_height,
            ctx.img_width,
            radii,
            conics,
            v_xys,
            v_conics,
        )
        return v_mean2d, v_scale, v_rot.view_as(rotation), None, None, None
