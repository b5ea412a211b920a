"""Tile-less Image-GS rendering — same API as the reference's
gsplat/rasterize_no_tiles.py:13-193."""

import torch
from torch import Tensor
from torch.autograd import Function

import gsplat.cuda as _C


def rasterize_gaussians_no_tiles(
    xys: Tensor, conics: Tensor, colors: Tensor, img_height: int, img_width: int
) -> Tensor:
    """Top-10 normalised weighted sum where every pixel considers all Gaussians."""
    if colors.dtype == torch.uint8:
        colors = colors.float() / 255
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise ValueError("xys must have dimensions (N, 2)")
    if colors.ndimension() != 2:
        raise ValueError("colors must have dimensions (N, D)")
    return _RasterizeGaussiansNoTiles.apply(
        xys.contiguous(), conics.contiguous(), colors.contiguous(), img_height, img_width
    )


class _RasterizeGaussiansNoTiles(Function):
    """Rasterizes 2D gaussians without tiles"""

    @staticmethod
    def forward(ctx, xys, conics, colors, img_height, img_width):
        num_points = xys.size(0)
        img_size = (img_width, img_height, 1)
        ctx.img_width = img_width
        ctx.img_height = img_height
        out_img, pixel_topk = _C.nd_rasterize_forward_no_tiles(
            img_size, num_points, xys, conics, colors
        )
        ctx.save_for_backward(xys, conics, colors, pixel_topk)
        return out_img

    @staticmethod
    def backward(ctx, v_out_img):
        xys, conics, colors, pixel_topk = ctx.saved_tensors
        v_xy, v_conic, v_colors = _C.nd_rasterize_backward_no_tiles(
            ctx.img_height, ctx.img_width, xys, conics, colors, v_out_img.contiguous(), pixel_topk
        )
        return v_xy, v_conic, v_colors, None, None


def rasterize_gaussians_simple(
    xys: Tensor, scale: Tensor, rot: Tensor, feat: Tensor, img_height: int, img_width: int
) -> Tensor:
    """Kept for API compatibility.  In the reference the kernels behind this
    function are commented out, so it renders zeros and returns zero gradients
    (gsplat/rasterize_no_tiles.py:102-193, gsplat/cuda/csrc/bindings.cu:2567-2681);
    this implementation preserves that behaviour."""
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise ValueError("xys must have dimensions (N, 2)")
    if feat.ndimension() != 2:
        raise ValueError("colors must have dimensions (N, D)")
    return _RasterizeGaussiansSimple.apply(
        xys.contiguous(), scale.contiguous(), rot.contiguous(), feat.contiguous(), img_height,
        img_width,
    )


class _RasterizeGaussiansSimple(Function):
    @staticmethod
    def forward(ctx, xys, scale, rot, feat, img_height, img_width):
        ctx.img_height = img_height
        ctx.img_width = img_width
        out_img, pixel_topk = _C.nd_rasterize_forward_simple(
            (img_width, img_height, 1), xys.size(0), xys, scale, rot, feat
        )
        ctx.save_for_backward(xys, scale, rot, feat, pixel_topk)
        return out_img

    @staticmethod
    def backward(ctx, v_out_img):
        xys, scale, rot, feat, pixel_topk = ctx.saved_tensors
        v_xy, v_scale, v_rot, v_feat = _C.nd_rasterize_backward_simple(
            ctx.img_height, ctx.img_width, xys, scale, rot, feat, v_out_img.contiguous(),
            pixel_topk,
        )
        return v_xy, v_scale, v_rot.view_as(rot), v_feat, None, None
