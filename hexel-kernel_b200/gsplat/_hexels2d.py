"""2D image-hexel entry points of ``gsplat.csrc`` (reference
gsplat/cuda/csrc/ext.cpp:14-65, bindings.h:143-555, bindings.cu:566-2457).

The reference binds sixteen functions — forward and backward of
{scale+rotation, affine} x {flat colour, colour gradient} x {scalar softness,
per-primitive softness}.  All sixteen keep their names, positional arguments
and returns here and dispatch to two C-ABI entry points
(hx_hexels2d_forward / hx_hexels2d_backward) whose templated sm_100a kernels
cover every variant.  An empty tensor means "absent", as in the reference.
"""

from __future__ import annotations

import torch

from ._lib import check_input, lib, ptr, stream, zero_views

TOP_K = 10


def _dims(t):
    return tuple(int(v) for v in t)


def _softness_stride(softnesses, num_points):
    if softnesses is None or softnesses.numel() == 0:
        return None, 0
    if softnesses.dtype != torch.float32:
        raise RuntimeError("softnesses must be float32")
    if softnesses.ndimension() == 1 and softnesses.size(0) == num_points:
        return softnesses.contiguous(), 1
    if softnesses.ndimension() == 2 and softnesses.size(0) == num_points and softnesses.size(1) == 3:
        return softnesses.contiguous(), 3
    raise RuntimeError("softnesses must have dimensions (num_points,) or (num_points, 3)")


def _emission(emission, num_points, channels):
    if emission is None or emission.numel() == 0:
        return None
    if emission.dtype != torch.float32:
        raise RuntimeError("emission must be float32")
    if emission.ndimension() != 2 or emission.size(0) != num_points or emission.size(1) != channels:
        raise RuntimeError("emission must have dimensions (num_points, channels)")
    return emission.contiguous()


def _check_color_grads(color_grads, channels):
    if color_grads.ndimension() != 3 or color_grads.size(1) != 2 or color_grads.size(2) != channels:
        raise RuntimeError("color_grads must have dimensions (num_points, 2, channels)")


def _check_affines(affines):
    if affines.ndimension() != 3 or affines.size(1) != 2 or affines.size(2) != 2:
        raise RuntimeError("affines must have dimensions (num_points, 2, 2)")


def _forward(tile_bounds, block, img_size, ids, bins, xys, colors, *, scales=None, rotation=None,
             affines=None, color_grads=None, color_grad_scale=0.0, aa_kernel_size=0.0,
             softnesses=None, softness_default=1.0, sharpness=None, emission=None):
    for t, n in ((ids, "gaussian_ids_sorted"), (bins, "tile_bins"), (xys, "xys")):
        check_input(t, n)
    if affines is None:
        check_input(scales, "scales")
        check_input(rotation, "rotation")
    else:
        _check_affines(affines)
    check_input(colors, "colors")
    b = _dims(block)
    if b[0] != 16 or b[1] != 16:
        raise RuntimeError(f"block must be (16, 16, 1); got {b}")
    tb, (w, h, _) = _dims(tile_bounds), _dims(img_size)
    channels = colors.size(1)
    n = xys.size(0)
    if color_grads is not None:
        check_input(color_grads, "color_grads")
        _check_color_grads(color_grads, channels)
    soft, stride = _softness_stride(softnesses, n)
    em = _emission(emission, n, channels)
    sh = None if sharpness is None or sharpness.numel() == 0 else sharpness.contiguous()
    dev = xys.device
    # the kernel writes every pixel when the tile grid is non-empty
    alloc = torch.empty if tb[0] > 0 and tb[1] > 0 else torch.zeros
    out_img = alloc((h, w, channels), dtype=torch.float32, device=dev)
    pixel_topk = alloc((h, w, TOP_K), dtype=torch.int32, device=dev)
    weights_sum = alloc((h, w), dtype=torch.float32, device=dev)
    entropy = alloc((h, w), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_hexels2d_forward", tb[0], tb[1], w, h, channels, n, ids.numel(), ptr(ids),
                 ptr(bins),
                 ptr(xys), ptr(scales), ptr(rotation), ptr(affines), ptr(colors),
                 ptr(color_grads), float(color_grad_scale), float(aa_kernel_size), ptr(soft),
                 stride, float(softness_default), ptr(sh), ptr(em), ptr(out_img),
                 ptr(pixel_topk), ptr(weights_sum), ptr(entropy), stream(dev))
    return out_img, pixel_topk, weights_sum, entropy


def _backward(img_height, img_width, block_h, block_w, xys, colors, v_output, v_weights_sum,
              v_entropy, pixel_topk, *, scales=None, rotation=None, affines=None,
              color_grads=None, color_grad_scale=0.0, aa_kernel_size=0.0, softnesses=None,
              softness_default=1.0, sharpness=None, emission=None, want_softness=False):
    check_input(xys, "xys")
    if affines is None:
        check_input(scales, "scales")
        check_input(rotation, "rotation")
    check_input(colors, "colors")
    if want_softness:
        check_input(softnesses, "softnesses")
    check_input(pixel_topk, "pixel_topk")
    check_input(v_weights_sum, "v_weights_sum")
    check_input(v_entropy, "v_entropy")
    if emission is not None:
        check_input(emission, "emission")
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise RuntimeError("xys must have dimensions (num_points, 2)")
    if affines is None:
        if scales.ndimension() != 2 or scales.size(1) != 2:
            raise RuntimeError("scales must have dimensions (num_points, 2)")
        if rotation.ndimension() != 2 or rotation.size(1) != 1:
            raise RuntimeError("rotation must have dimensions (num_points, 1)")
    else:
        _check_affines(affines)
    if colors.ndimension() != 2:
        raise RuntimeError("colors must have 2 dimensions")
    if int(block_h) != 16 or int(block_w) != 16:
        raise RuntimeError("BLOCK_H/BLOCK_W must be 16/16")
    n, channels, dev = xys.size(0), colors.size(1), xys.device
    if color_grads is not None:
        _check_color_grads(color_grads, channels)
    soft, stride = _softness_stride(softnesses, n)
    em = _emission(emission, n, channels)
    sh = None if sharpness is None or sharpness.numel() == 0 else sharpness.contiguous()
    # all gradient outputs zeroed by one fill of one allocation
    shapes = {"v_xy": (n, 2), "v_colors": (n, channels), "v_sharpness": (n, 1),
              "v_emission": tuple(emission.shape) if emission is not None else (0,)}
    if affines is None:
        shapes.update(v_scale=(n, 2), v_rot=(n, 1))
    else:
        shapes.update(v_affines=(n, 2, 2))
    if color_grads is not None:
        shapes.update(v_color_grads=(n, 2, channels))
    if softnesses is not None:
        shapes.update(v_softnesses=tuple(softnesses.shape))
    g = dict(zip(shapes, zero_views(dev, list(shapes.values()))))
    v_xy, v_colors, v_sharpness, v_emission = (g["v_xy"], g["v_colors"], g["v_sharpness"],
                                               g["v_emission"])
    v_scale, v_rot, v_affines = g.get("v_scale"), g.get("v_rot"), g.get("v_affines")
    v_color_grads, v_softnesses = g.get("v_color_grads"), g.get("v_softnesses")
    with torch.cuda.device(dev):
        lib.call("hx_hexels2d_backward", int(img_width), int(img_height), channels, n, ptr(xys),
                 ptr(scales), ptr(rotation), ptr(affines), ptr(colors), ptr(color_grads),
                 float(color_grad_scale), ptr(em), ptr(v_output.contiguous()),
                 ptr(v_weights_sum), ptr(v_entropy), ptr(pixel_topk), float(aa_kernel_size),
                 ptr(soft), stride, float(softness_default), ptr(sh), ptr(v_xy), ptr(v_scale),
                 ptr(v_rot), ptr(v_affines), ptr(v_colors), ptr(v_color_grads),
                 ptr(v_emission) if em is not None else None, ptr(v_sharpness),
                 ptr(v_softnesses) if soft is not None else None, stream(dev))
    return dict(v_xy=v_xy, v_scale=v_scale, v_rot=v_rot, v_affines=v_affines, v_colors=v_colors,
                v_color_grads=v_color_grads, v_emission=v_emission, v_sharpness=v_sharpness,
                v_softnesses=v_softnesses)


# ---- forward (bindings.h:143-555) ------------------------------------------------
def nd_rasterize_forward_topk_norm_hexels(tile_bounds, block, img_size, gaussian_ids_sorted,
                                          tile_bins, xys, scales, rotation, colors,
                                          aa_kernel_size, softness, sharpness, emission):
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    scales=scales, rotation=rotation, aa_kernel_size=aa_kernel_size,
                    softness_default=softness, sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_softness(tile_bounds, block, img_size,
                                                   gaussian_ids_sorted, tile_bins, xys, scales,
                                                   rotation, colors, aa_kernel_size, softnesses,
                                                   softness_default, sharpness, emission):
    check_input(softnesses, "softnesses")
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    scales=scales, rotation=rotation, aa_kernel_size=aa_kernel_size,
                    softnesses=softnesses, softness_default=softness_default,
                    sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_color_grad(tile_bounds, block, img_size,
                                                     gaussian_ids_sorted, tile_bins, xys, scales,
                                                     rotation, colors, color_grads,
                                                     color_grad_scale, aa_kernel_size, softness,
                                                     sharpness, emission):
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    scales=scales, rotation=rotation, color_grads=color_grads,
                    color_grad_scale=color_grad_scale, aa_kernel_size=aa_kernel_size,
                    softness_default=softness, sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_color_grad_softness(
        tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, scales, rotation,
        colors, color_grads, color_grad_scale, aa_kernel_size, softnesses, softness_default,
        sharpness, emission):
    check_input(softnesses, "softnesses")
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    scales=scales, rotation=rotation, color_grads=color_grads,
                    color_grad_scale=color_grad_scale, aa_kernel_size=aa_kernel_size,
                    softnesses=softnesses, softness_default=softness_default,
                    sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_affine(tile_bounds, block, img_size,
                                                 gaussian_ids_sorted, tile_bins, xys, affines,
                                                 colors, aa_kernel_size, softness, sharpness,
                                                 emission):
    check_input(affines, "affines")
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    affines=affines, aa_kernel_size=aa_kernel_size, softness_default=softness,
                    sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_affine_softness(
        tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, affines, colors,
        aa_kernel_size, softnesses, softness_default, sharpness, emission):
    check_input(affines, "affines")
    check_input(softnesses, "softnesses")
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    affines=affines, aa_kernel_size=aa_kernel_size, softnesses=softnesses,
                    softness_default=softness_default, sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_affine_color_grad(
        tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, affines, colors,
        color_grads, color_grad_scale, aa_kernel_size, softness, sharpness, emission):
    check_input(affines, "affines")
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    affines=affines, color_grads=color_grads, color_grad_scale=color_grad_scale,
                    aa_kernel_size=aa_kernel_size, softness_default=softness,
                    sharpness=sharpness, emission=emission)


def nd_rasterize_forward_topk_norm_hexels_affine_color_grad_softness(
        tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, affines, colors,
        color_grads, color_grad_scale, aa_kernel_size, softnesses, softness_default, sharpness,
        emission):
    check_input(affines, "affines")
    check_input(softnesses, "softnesses")
    check_input(emission, "emission")
    return _forward(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, colors,
                    affines=affines, color_grads=color_grads, color_grad_scale=color_grad_scale,
                    aa_kernel_size=aa_kernel_size, softnesses=softnesses,
                    softness_default=softness_default, sharpness=sharpness, emission=emission)


# ---- backward --------------------------------------------------------------------
def nd_rasterize_backward_topk_norm_hexels(img_height, img_width, BLOCK_H, BLOCK_W,
                                           gaussians_ids_sorted, tile_bins, xys, scales,
                                           rotation, colors, v_output, v_weights_sum, v_entropy,
                                           pixel_topk, aa_kernel_size, softness, sharpness,
                                           emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, scales=scales, rotation=rotation,
                  aa_kernel_size=aa_kernel_size, softness_default=softness, sharpness=sharpness,
                  emission=emission)
    return r["v_xy"], r["v_scale"], r["v_rot"], r["v_colors"], r["v_emission"], r["v_sharpness"]


def nd_rasterize_backward_topk_norm_hexels_softness(img_height, img_width, BLOCK_H, BLOCK_W,
                                                    gaussians_ids_sorted, tile_bins, xys, scales,
                                                    rotation, colors, softnesses, v_output,
                                                    v_weights_sum, v_entropy, pixel_topk,
                                                    aa_kernel_size, softness_default, sharpness,
                                                    emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, scales=scales, rotation=rotation,
                  aa_kernel_size=aa_kernel_size, softnesses=softnesses,
                  softness_default=softness_default, sharpness=sharpness, emission=emission,
                  want_softness=True)
    return (r["v_xy"], r["v_scale"], r["v_rot"], r["v_colors"], r["v_emission"],
            r["v_sharpness"], r["v_softnesses"])


def nd_rasterize_backward_topk_norm_hexels_color_grad(img_height, img_width, BLOCK_H, BLOCK_W,
                                                      gaussians_ids_sorted, tile_bins, xys,
                                                      scales, rotation, colors, color_grads,
                                                      color_grad_scale, v_output, v_weights_sum,
                                                      v_entropy, pixel_topk, aa_kernel_size,
                                                      softness, sharpness, emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, scales=scales, rotation=rotation,
                  color_grads=color_grads, color_grad_scale=color_grad_scale,
                  aa_kernel_size=aa_kernel_size, softness_default=softness, sharpness=sharpness,
                  emission=emission)
    return (r["v_xy"], r["v_scale"], r["v_rot"], r["v_colors"], r["v_color_grads"],
            r["v_emission"], r["v_sharpness"])


def nd_rasterize_backward_topk_norm_hexels_color_grad_softness(
        img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted, tile_bins, xys, scales,
        rotation, colors, color_grads, softnesses, color_grad_scale, v_output, v_weights_sum,
        v_entropy, pixel_topk, aa_kernel_size, softness_default, sharpness, emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, scales=scales, rotation=rotation,
                  color_grads=color_grads, color_grad_scale=color_grad_scale,
                  aa_kernel_size=aa_kernel_size, softnesses=softnesses,
                  softness_default=softness_default, sharpness=sharpness, emission=emission,
                  want_softness=True)
    return (r["v_xy"], r["v_scale"], r["v_rot"], r["v_colors"], r["v_color_grads"],
            r["v_emission"], r["v_sharpness"], r["v_softnesses"])


def nd_rasterize_backward_topk_norm_hexels_affine(img_height, img_width, BLOCK_H, BLOCK_W,
                                                  gaussians_ids_sorted, tile_bins, xys, affines,
                                                  colors, v_output, v_weights_sum, v_entropy,
                                                  pixel_topk, aa_kernel_size, softness,
                                                  sharpness, emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, affines=affines, aa_kernel_size=aa_kernel_size,
                  softness_default=softness, sharpness=sharpness, emission=emission)
    return r["v_xy"], r["v_affines"], r["v_colors"], r["v_emission"], r["v_sharpness"]


def nd_rasterize_backward_topk_norm_hexels_affine_softness(
        img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted, tile_bins, xys, affines,
        colors, softnesses, v_output, v_weights_sum, v_entropy, pixel_topk, aa_kernel_size,
        softness_default, sharpness, emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, affines=affines, aa_kernel_size=aa_kernel_size,
                  softnesses=softnesses, softness_default=softness_default, sharpness=sharpness,
                  emission=emission, want_softness=True)
    return (r["v_xy"], r["v_affines"], r["v_colors"], r["v_emission"], r["v_sharpness"],
            r["v_softnesses"])


def nd_rasterize_backward_topk_norm_hexels_affine_color_grad(
        img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted, tile_bins, xys, affines,
        colors, color_grads, color_grad_scale, v_output, v_weights_sum, v_entropy, pixel_topk,
        aa_kernel_size, softness, sharpness, emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, affines=affines, color_grads=color_grads,
                  color_grad_scale=color_grad_scale, aa_kernel_size=aa_kernel_size,
                  softness_default=softness, sharpness=sharpness, emission=emission)
    return (r["v_xy"], r["v_affines"], r["v_colors"], r["v_color_grads"], r["v_emission"],
            r["v_sharpness"])


def nd_rasterize_backward_topk_norm_hexels_affine_color_grad_softness(
        img_height, img_width, BLOCK_H, BLOCK_W, gaussians_ids_sorted, tile_bins, xys, affines,
        colors, color_grads, softnesses, color_grad_scale, v_output, v_weights_sum, v_entropy,
        pixel_topk, aa_kernel_size, softness_default, sharpness, emission):
    r = _backward(img_height, img_width, BLOCK_H, BLOCK_W, xys, colors, v_output, v_weights_sum,
                  v_entropy, pixel_topk, affines=affines, color_grads=color_grads,
                  color_grad_scale=color_grad_scale, aa_kernel_size=aa_kernel_size,
                  softnesses=softnesses, softness_default=softness_default, sharpness=sharpness,
                  emission=emission, want_softness=True)
    return (r["v_xy"], r["v_affines"], r["v_colors"], r["v_color_grads"], r["v_emission"],
            r["v_sharpness"], r["v_softnesses"])


_NAMES = [n for n in list(globals()) if n.startswith("nd_rasterize_")]


def exports() -> dict:
    return {n: globals()[n] for n in _NAMES}
