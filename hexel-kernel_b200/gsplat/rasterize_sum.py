"""Image-GS tile rasterisation — same API as the reference's
gsplat/rasterize_sum.py:14-226.

Forward: prefix sum of tile counts (one 8-byte device-to-host read of the
total, as the reference's ``.item()``), fused binning (emit 32-bit tile keys,
stable radix sort of ceil(log2(tiles)) bits, tile ranges), then compositing.
``topk_norm=True`` keeps the 10 largest weights per pixel and normalises
them; ``False`` is the plain weighted sum.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor
from torch.autograd import Function

import gsplat.cuda as _C
from .utils import bin_gaussians_fused, compute_cumulative_intersects, count_tiles_in_rows


def rasterize_gaussians_sum(
    xys: Tensor,
    radii: Tensor,
    conics: Tensor,
    num_tiles_hit: Tensor,
    colors: Tensor,
    img_height: int,
    img_width: int,
    BLOCK_H: int = 16,
    BLOCK_W: int = 16,
    topk_norm: bool = False,
    *,
    tile_rows: Optional[Tuple[int, int]] = None,
) -> Tensor:
    """Render (H, W, C) from projected 2D Gaussians.

    `tile_rows=(begin, end)` (keyword only, not in the reference) renders only
    that horizontal stripe of 16-pixel tile rows; pixels outside it are zero
    and receive no gradient.  It is how one image is sharded over GPUs."""
    if colors.dtype == torch.uint8:
        colors = colors.float() / 255
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise ValueError("xys must have dimensions (N, 2)")
    if colors.ndimension() != 2:
        raise ValueError("colors must have dimensions (N, D)")
    return _RasterizeGaussiansSum.apply(
        xys.contiguous(),
        radii.contiguous(),
        conics.contiguous(),
        num_tiles_hit.contiguous(),
        colors.contiguous(),
        img_height,
        img_width,
        BLOCK_H,
        BLOCK_W,
        topk_norm,
        tile_rows,
    )


class _RasterizeGaussiansSum(Function):
    """Rasterizes 2D gaussians"""

    @staticmethod
    def forward(ctx, xys, radii, conics, num_tiles_hit, colors, img_height, img_width,
                BLOCK_H=16, BLOCK_W=16, topk_norm=False, tile_rows=None):
        num_points = xys.size(0)
        tile_bounds = (
            (img_width + BLOCK_W - 1) // BLOCK_W,
            (img_height + BLOCK_H - 1) // BLOCK_H,
            1,
        )
        block = (BLOCK_W, BLOCK_H, 1)
        img_size = (img_width, img_height, 1)
        if tile_rows is not None:
            num_tiles_hit = count_tiles_in_rows(xys, radii, tile_bounds, tile_rows)
        num_intersects, cum_tiles_hit = compute_cumulative_intersects(num_tiles_hit)
        gaussian_ids_sorted, tile_bins = bin_gaussians_fused(
            num_points, num_intersects, xys, radii, cum_tiles_hit, tile_bounds, tile_rows
        )

        ctx.img_width = img_width
        ctx.img_height = img_height
        ctx.BLOCK_H = BLOCK_H
        ctx.BLOCK_W = BLOCK_W
        ctx.num_intersects = num_intersects
        ctx.topk_norm = topk_norm
        # a stripe's pixels outside its rows hold no ids: the backward skips them
        ctx.rows = (None if tile_rows is None else
                    (tile_rows[0] * BLOCK_H, min(tile_rows[1] * BLOCK_H, img_height)))

        if not topk_norm:
            (out_img,) = _C.nd_rasterize_forward(
                tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, conics, colors
            )
            ctx.save_for_backward(gaussian_ids_sorted, tile_bins, xys, conics, colors)
        else:
            out_img, pixel_topk = _C.nd_rasterize_forward_topk_norm(
                tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, conics, colors
            )
            ctx.save_for_backward(gaussian_ids_sorted, tile_bins, xys, conics, colors, pixel_topk)
        return out_img

    @staticmethod
    def backward(ctx, v_out_img):
        v_out_img = v_out_img.contiguous()
        if not ctx.topk_norm:
            gaussian_ids_sorted, tile_bins, xys, conics, colors = ctx.saved_tensors
            v_xy, v_conic, v_colors = _C.nd_rasterize_backward(
                ctx.img_height, ctx.img_width, ctx.BLOCK_H, ctx.BLOCK_W, gaussian_ids_sorted,
                tile_bins, xys, conics, colors, v_out_img,
            )
        else:
            gaussian_ids_sorted, tile_bins, xys, conics, colors, pixel_topk = ctx.saved_tensors
            v_xy, v_conic, v_colors = _C.nd_rasterize_backward_topk_norm(
                ctx.img_height, ctx.img_width, ctx.BLOCK_H, ctx.BLOCK_W, gaussian_ids_sorted,
                tile_bins, xys, conics, colors, v_out_img, pixel_topk, rows=ctx.rows,
            )
        return (v_xy, None, v_conic, None, v_colors, None, None, None, None, None, None)
