"""``gsplat.csrc`` — the 2D extension module of the reference, re-implemented.

Same function names, positional arguments, return tuples, dtypes and error
messages as the reference's pybind module (gsplat/cuda/csrc/ext.cpp:4-83,
bindings.h), but each function is a thin host wrapper: it checks and
allocates with PyTorch on the inputs' device and launches the hand-written
sm_100a kernels of ``libhexel_b200.so`` on the current stream through the
C-ABI.  Unlike the reference it does not synchronise the device after every
launch and raises ``RuntimeError`` instead of exiting on a CUDA error.
"""

from __future__ import annotations

from typing import Tuple

import torch

from ._lib import check_input, lib, ptr, stream, workspace, zero_views
from . import _hexels2d

TOP_K = 10
BLOCK_X = 16
BLOCK_Y = 16


def _dims(t) -> Tuple[int, int, int]:
    t = tuple(int(v) for v in t)
    if len(t) != 3:
        raise TypeError("expected a 3-tuple of ints")
    return t


def _check_block(block) -> None:
    b = _dims(block)
    if b[0] != BLOCK_X or b[1] != BLOCK_Y:
        raise RuntimeError(f"block must be ({BLOCK_X}, {BLOCK_Y}, 1); got {b}")


def _tile_bounds_for(img_height: int, img_width: int, block_h: int, block_w: int):
    if block_h != BLOCK_Y or block_w != BLOCK_X:
        raise RuntimeError(f"BLOCK_H/BLOCK_W must be {BLOCK_Y}/{BLOCK_X}")
    return (img_width + BLOCK_X - 1) // BLOCK_X, (img_height + BLOCK_Y - 1) // BLOCK_Y


# --------------------------------------------------------------------------
# S1 projection (bindings.cu:2746-2846) and utilities (bindings.cu:20-116)
# --------------------------------------------------------------------------
def project_gaussians_2d_scale_rot_forward(num_points, means2d, scales2d, rotation, img_height,
                                           img_width, tile_bounds):
    check_input(means2d, "means2d")
    means2d = means2d.contiguous()
    scales2d = scales2d.contiguous()
    rotation = rotation.contiguous()
    dev = means2d.device
    tb = _dims(tile_bounds)
    n = int(num_points)
    opts = dict(device=dev)
    xys = torch.empty((n, 2), dtype=torch.float32, **opts)
    radii = torch.empty((n,), dtype=torch.int32, **opts)
    conics = torch.empty((n, 3), dtype=torch.float32, **opts)
    num_tiles_hit = torch.empty((n,), dtype=torch.int32, **opts)
    with torch.cuda.device(dev):
        lib.call("hx_project_gaussians_2d_scale_rot_forward", n, ptr(means2d), ptr(scales2d),
                 ptr(rotation), int(img_height), int(img_width), tb[0], tb[1], ptr(xys),
                 ptr(radii), ptr(conics), ptr(num_tiles_hit), stream(dev))
    return xys, radii, conics, num_tiles_hit


def project_gaussians_2d_scale_rot_backward(num_points, means2d, scales2d, rotation, img_height,
                                            img_width, radii, conics, v_xy, v_conic):
    check_input(means2d, "means2d")
    dev = means2d.device
    n = int(num_points)
    scales2d, rotation = scales2d.contiguous(), rotation.contiguous()
    radii, conics = radii.contiguous(), conics.contiguous()
    v_xy, v_conic = v_xy.contiguous(), v_conic.contiguous()
    v_cov2d = torch.empty((n, 3), dtype=torch.float32, device=dev)
    v_scale = torch.empty((n, 2), dtype=torch.float32, device=dev)
    v_rot = torch.empty((n, 1), dtype=torch.float32, device=dev)
    v_mean2d = torch.empty((n, 2), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_project_gaussians_2d_scale_rot_backward", n, ptr(means2d), ptr(scales2d),
                 ptr(rotation), int(img_height), int(img_width), ptr(radii), ptr(conics),
                 ptr(v_xy), ptr(v_conic), ptr(v_cov2d), ptr(v_mean2d), ptr(v_scale), ptr(v_rot),
                 stream(dev))
    return v_cov2d, v_mean2d, v_scale, v_rot


def compute_cov2d_bounds(num_pts, covs2d):
    check_input(covs2d, "covs2d")
    n = int(num_pts)
    dev = covs2d.device
    conics = torch.zeros((n, covs2d.size(1)), dtype=torch.float32, device=dev)
    radii = torch.zeros((n, 1), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_compute_cov2d_bounds", n, ptr(covs2d), ptr(conics), ptr(radii), stream(dev))
    return conics, radii


def map_gaussian_to_intersects(num_points, num_intersects, xys, radii, cum_tiles_hit,
                               tile_bounds):
    check_input(xys, "xys")
    check_input(radii, "radii")
    check_input(cum_tiles_hit, "cum_tiles_hit")
    dev = xys.device
    tb = _dims(tile_bounds)
    ni = int(num_intersects)
    gaussian_ids = torch.zeros((ni,), dtype=torch.int32, device=dev)
    isect_ids = torch.zeros((ni,), dtype=torch.int64, device=dev)
    radii32 = radii.to(torch.int32).contiguous()
    cum32 = cum_tiles_hit.to(torch.int32).contiguous()
    with torch.cuda.device(dev):
        lib.call("hx_map_gaussian_to_intersects", int(num_points), ni, ptr(xys), ptr(radii32),
                 ptr(cum32), tb[0], tb[1], ptr(isect_ids), ptr(gaussian_ids), stream(dev))
    return isect_ids, gaussian_ids


def get_tile_bin_edges(num_intersects, num_tiles, isect_ids_sorted):
    check_input(isect_ids_sorted, "isect_ids_sorted")
    dev = isect_ids_sorted.device
    tile_bins = torch.empty((int(num_tiles), 2), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_get_tile_bin_edges", int(num_intersects), int(num_tiles),
                 ptr(isect_ids_sorted), ptr(tile_bins), stream(dev))
    return tile_bins


# --------------------------------------------------------------------------
# S3 Image-GS compositing (bindings.cu:118-565, 2683-2744)
# --------------------------------------------------------------------------
def _raster_inputs(gaussian_ids_sorted, tile_bins, xys, conics, colors):
    check_input(gaussian_ids_sorted, "gaussian_ids_sorted")
    check_input(tile_bins, "tile_bins")
    check_input(xys, "xys")
    check_input(conics, "conics")
    check_input(colors, "colors")
    if gaussian_ids_sorted.dtype != torch.int32 or tile_bins.dtype != torch.int32:
        raise RuntimeError("gaussian_ids_sorted and tile_bins must be int32")


def nd_rasterize_forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys,
                         conics, colors):
    _raster_inputs(gaussian_ids_sorted, tile_bins, xys, conics, colors)
    _check_block(block)
    tb, (w, h, _) = _dims(tile_bounds), _dims(img_size)
    channels = colors.size(1)
    dev = xys.device
    out_img = torch.zeros((h, w, channels), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_nd_rasterize_forward", tb[0], tb[1], w, h, channels, xys.size(0),
                 gaussian_ids_sorted.numel(), ptr(gaussian_ids_sorted), ptr(tile_bins), ptr(xys), ptr(conics), ptr(colors),
                 ptr(out_img), stream(dev))
    return (out_img,)


def rasterize_forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, conics,
                      colors):
    if colors.ndimension() != 2 or colors.size(1) != 3:
        raise RuntimeError("colors must have dimensions (num_points, 3)")
    return nd_rasterize_forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys,
                                conics, colors)


def _check_xys_colors(xys, colors):
    check_input(xys, "xys")
    check_input(colors, "colors")
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise RuntimeError("xys must have dimensions (num_points, 2)")
    if colors.ndimension() != 2:
        raise RuntimeError("colors must have 2 dimensions")


def nd_rasterize_backward(img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted,
                          tile_bins, xys, conics, colors, v_output):
    _check_xys_colors(xys, colors)
    tx, ty = _tile_bounds_for(int(img_height), int(img_width), int(BLOCK_H), int(BLOCK_W))
    n, channels, dev = xys.size(0), colors.size(1), xys.device
    v_xy, v_conic, v_colors = zero_views(dev, [(n, 2), (n, 3), (n, channels)])
    v_output = v_output.contiguous()
    with torch.cuda.device(dev):
        lib.call("hx_nd_rasterize_backward", tx, ty, int(img_width), int(img_height), channels,
                 n, gaussians_ids_sorted.numel(), ptr(gaussians_ids_sorted.contiguous()), ptr(tile_bins.contiguous()), ptr(xys),
                 ptr(conics.contiguous()), ptr(colors), ptr(v_output), ptr(v_xy), ptr(v_conic),
                 ptr(v_colors), stream(dev))
    return v_xy, v_conic, v_colors


def rasterize_backward(img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted, tile_bins,
                       xys, conics, colors, v_output):
    if colors.ndimension() != 2 or colors.size(1) != 3:
        raise RuntimeError("colors must have 2 dimensions")
    return nd_rasterize_backward(img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted,
                                 tile_bins, xys, conics, colors, v_output)


def _topk_forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, conics,
                  colors, stats: bool):
    _raster_inputs(gaussian_ids_sorted, tile_bins, xys, conics, colors)
    _check_block(block)
    tb, (w, h, _) = _dims(tile_bounds), _dims(img_size)
    channels = colors.size(1)
    dev = xys.device
    # the kernel writes every pixel when the tile grid is non-empty
    alloc = torch.empty if tb[0] > 0 and tb[1] > 0 else torch.zeros
    out_img = alloc((h, w, channels), dtype=torch.float32, device=dev)
    pixel_topk = alloc((h, w, TOP_K), dtype=torch.int32, device=dev)
    weights_sum = alloc((h, w), dtype=torch.float32, device=dev) if stats else None
    entropy = alloc((h, w), dtype=torch.float32, device=dev) if stats else None
    with torch.cuda.device(dev):
        lib.call("hx_nd_rasterize_forward_topk_norm", tb[0], tb[1], w, h, channels, xys.size(0),
                 gaussian_ids_sorted.numel(), ptr(gaussian_ids_sorted), ptr(tile_bins), ptr(xys), ptr(conics), ptr(colors),
                 ptr(out_img), ptr(pixel_topk), ptr(weights_sum), ptr(entropy), stream(dev))
    if stats:
        return out_img, pixel_topk, weights_sum, entropy
    return out_img, pixel_topk


def nd_rasterize_forward_topk_norm(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins,
                                   xys, conics, colors):
    return _topk_forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys,
                         conics, colors, stats=False)


def nd_rasterize_forward_topk_norm_stats(tile_bounds, block, img_size, gaussian_ids_sorted,
                                         tile_bins, xys, conics, colors):
    return _topk_forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys,
                         conics, colors, stats=True)


def _topk_backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, conics, colors, v_output,
                   v_weights_sum, v_entropy, pixel_topk, rows=None):
    _check_xys_colors(xys, colors)
    check_input(pixel_topk, "pixel_topk")
    _tile_bounds_for(int(img_height), int(img_width), int(BLOCK_H), int(BLOCK_W))
    n, channels, dev = xys.size(0), colors.size(1), xys.device
    v_xy, v_conic, v_colors = zero_views(dev, [(n, 2), (n, 3), (n, channels)])
    v_output = v_output.contiguous()
    args = (int(img_width), int(img_height), channels, n, ptr(xys), ptr(conics.contiguous()),
            ptr(colors), ptr(v_output), ptr(v_weights_sum), ptr(v_entropy), ptr(pixel_topk))
    outs = (ptr(v_xy), ptr(v_conic), ptr(v_colors), stream(dev))
    with torch.cuda.device(dev):
        if rows is None:
            lib.call("hx_nd_rasterize_backward_topk_norm", *args, *outs)
        else:
            lib.call("hx_nd_rasterize_backward_topk_norm_rows", *args, int(rows[0]),
                     int(rows[1]), *outs)
    return v_xy, v_conic, v_colors


def nd_rasterize_backward_topk_norm(img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted,
                                    tile_bins, xys, conics, colors, v_output, pixel_topk, *,
                                    rows=None):
    """The reference's top-K backward.  `rows=(begin, end)` (keyword only,
    not in the reference) back-propagates pixel rows [begin, end) only: the
    backward of one stripe, whose upstream gradient is zero elsewhere."""
    return _topk_backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, conics, colors, v_output,
                          None, None, pixel_topk, rows)


def nd_rasterize_backward_topk_norm_stats(img_height, img_width, BLOCK_H, BLOCK_W,
                                          gaussians_ids_sorted, tile_bins, xys, conics, colors,
                                          v_output, v_weights_sum, v_entropy, pixel_topk):
    check_input(v_weights_sum, "v_weights_sum")
    check_input(v_entropy, "v_entropy")
    return _topk_backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, conics, colors, v_output,
                          v_weights_sum, v_entropy, pixel_topk)


# --------------------------------------------------------------------------
# S4 tile-less rendering (bindings.cu:2459-2681)
# --------------------------------------------------------------------------
def nd_rasterize_forward_no_tiles(img_size, num_points, xys, conics, colors):
    check_input(xys, "xys")
    check_input(conics, "conics")
    check_input(colors, "colors")
    w, h, _ = _dims(img_size)
    channels, dev = colors.size(1), xys.device
    out_img = torch.zeros((h, w, channels), dtype=torch.float32, device=dev)
    pixel_topk = torch.zeros((h, w, TOP_K), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_nd_rasterize_forward_no_tiles", w, h, channels, int(num_points), ptr(xys),
                 ptr(conics), ptr(colors), ptr(out_img), ptr(pixel_topk), stream(dev))
    return out_img, pixel_topk


def nd_rasterize_backward_no_tiles(img_height, img_width, xys, conics, colors, v_output,
                                   pixel_topk):
    _check_xys_colors(xys, colors)
    check_input(pixel_topk, "pixel_topk")
    n, channels, dev = xys.size(0), colors.size(1), xys.device
    v_xy = torch.zeros((n, 2), dtype=torch.float32, device=dev)
    v_conic = torch.zeros((n, 3), dtype=torch.float32, device=dev)
    v_colors = torch.zeros((n, channels), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_nd_rasterize_backward_no_tiles", int(img_width), int(img_height), channels,
                 n, ptr(xys), ptr(conics.contiguous()), ptr(colors), ptr(v_output.contiguous()),
                 ptr(pixel_topk), ptr(v_xy), ptr(v_conic), ptr(v_colors), stream(dev))
    return v_xy, v_conic, v_colors


def nd_rasterize_forward_simple(img_size, num_points, xys, scale, rot, feat):
    """The reference binds this entry point but launches no kernel: it returns
    zero-filled outputs (gsplat/cuda/csrc/bindings.cu:2567-2617).  Kept as is."""
    for t, name in ((xys, "xys"), (scale, "scale"), (rot, "rot"), (feat, "feat")):
        check_input(t, name)
    w, h, _ = _dims(img_size)
    dev = xys.device
    return (torch.zeros((h, w, feat.size(1)), dtype=torch.float32, device=dev),
            torch.zeros((h, w, TOP_K), dtype=torch.int32, device=dev))


def nd_rasterize_backward_simple(img_height, img_width, xys, scale, rot, feat, v_output,
                                 pixel_topk):
    """Zero gradients, as the reference stub (gsplat/cuda/csrc/bindings.cu:2620-2681)."""
    for t, name in ((xys, "xys"), (scale, "scale"), (rot, "rot"), (feat, "feat"),
                    (pixel_topk, "pixel_topk")):
        check_input(t, name)
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise RuntimeError("xys must have dimensions (num_points, 2)")
    if feat.ndimension() != 2:
        raise RuntimeError("colors must have 2 dimensions")
    n, dev = xys.size(0), xys.device
    z = lambda *s: torch.zeros(s, dtype=torch.float32, device=dev)  # noqa: E731
    return z(n, 2), z(n, 2), z(n, 1), z(n, feat.size(1))


# --------------------------------------------------------------------------
# S5 2D image hexels (bindings.cu:566-2457) — see _hexels2d.py
# --------------------------------------------------------------------------
globals().update(_hexels2d.exports())
