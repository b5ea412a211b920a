"""``gsplat.cuda_hexels3d._C`` — the 3D hexel surfel rasteriser module.

Same function names, positional arguments, return tuples and checks as the
reference's extension (gsplat/cuda_hexels3d/csrc/ext.cpp:5-23,
hexels3d_forward.h, hexels3d_backward.h); each function drives the sm_100a
kernels of ``libhexel_b200.so`` through its C-ABI on PyTorch's current stream:

  preprocess -> prefix sum (one 8-byte read-back of the intersection count,
  as the reference) -> emit (tile|depth) keys -> stable radix sort -> tile
  ranges -> compositing; backward: reverse traversal -> geometry VJP.

The cached forward returns the reference's eleven saved buffers, and the
cached backward accepts them.  The diagnostic exact-sort / pixel-risk oracles
of the reference are not part of the training or render path and are not
provided by this build.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .._lib import check_input, lib, ptr, stream, workspace, zero_views

kNumChannels = 3
_EMPTY_CACHE: dict = {}

# Optional callable invoked with a stage name after each stage's launches
# ("preprocess", "scan", "bin", "render_fwd", "render_bwd", "geometry_bwd"),
# e.g. to record CUDA events between stages.  None in normal use.
stage_hook = None


def _mark(name: str) -> None:
    if stage_hook is not None:
        stage_hook(name)


def _zero_views(dev, shapes):
    return zero_views(dev, shapes)


def _empty(x: torch.Tensor, dtype=None) -> torch.Tensor:
    return torch.empty((0,), device=x.device, dtype=dtype or x.dtype)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _checks(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
            specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix, campos,
            background, image_width, image_height, softness, color_model, view_model,
            use_view_grads):
    """The reference's argument checks (hexels3d_forward.cu:2724-2857)."""
    names = ("means3d", "scales", "rotations", "colors", "color_grads", "color_quads",
             "view_grads", "specular_ks", "specular_log_s", "opacities", "softnesses",
             "viewmatrix", "projmatrix", "campos", "background")
    tensors = (means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
               specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix,
               campos, background)
    for t, n in zip(tensors, names):
        check_input(t, n)
    _check(means3d.ndimension() == 2 and means3d.size(1) == 3, "means3d must have shape (P,3)")
    _check(scales.ndimension() == 2 and scales.size(1) == 2, "scales must have shape (P,2)")
    _check(rotations.ndimension() == 2 and rotations.size(1) == 4,
           "rotations must have shape (P,4)")
    _check(colors.ndimension() == 2 and colors.size(1) == 3, "colors must have shape (P,3)")
    _check(0 <= color_model <= 3,
           "color_model must be one of: 0 (flat), 1 (linear), 2 (quadratic), 3 (quadratic_bounded)")
    _check(0 <= view_model <= 2, "view_model must be one of: 0 (none), 1 (linear), 2 (lobe)")
    P = means3d.size(0)
    want_linear = color_model >= 1
    want_quad = color_model in (2, 3)
    cg_ok = color_grads.ndimension() == 3 and color_grads.size(1) == 2 and color_grads.size(2) == 3
    if want_linear:
        _check(cg_ok, "color_grads must have shape (P,2,3)")
        _check(color_grads.size(0) == P, "color_grads must have shape (P,2,3)")
    else:
        _check(color_grads.numel() == 0 or cg_ok, "color_grads must have shape (P,2,3) or be empty")
    cq_ok = color_quads.ndimension() == 3 and color_quads.size(1) == 3 and color_quads.size(2) == 3
    if want_quad:
        _check(cq_ok, "color_quads must have shape (P,3,3)")
        _check(color_quads.size(0) == P, "color_quads must have shape (P,3,3)")
    else:
        _check(color_quads.numel() == 0 or cq_ok, "color_quads must have shape (P,3,3) or be empty")
    vg_ok = view_grads.ndimension() == 3 and view_grads.size(1) == 3 and view_grads.size(2) == 3
    if use_view_grads:
        _check(vg_ok, "view_grads must have shape (P,3,3)")
        _check(view_grads.size(0) == P, "view_grads must have shape (P,3,3)")
    else:
        _check(view_grads.numel() == 0 or vg_ok, "view_grads must have shape (P,3,3) or be empty")
    if view_model == 2:
        _check(specular_ks.ndimension() == 2 and specular_ks.size(1) == 3,
               "specular_ks must have shape (P,3)")
        _check(specular_log_s.ndimension() == 1, "specular_log_s must have shape (P,)")
        _check(specular_ks.size(0) == P, "specular_ks must have shape (P,3)")
        _check(specular_log_s.numel() == P, "specular_log_s must have shape (P,)")
    _check(opacities.ndimension() == 1, "opacities must have shape (P,)")
    _check(softnesses.ndimension() in (1, 2), "softnesses must have shape (P,), (P,3) or (0,)")
    _check(viewmatrix.numel() == 16, "viewmatrix must have 16 elements")
    _check(projmatrix.numel() == 16, "projmatrix must have 16 elements")
    _check(campos.numel() == 3, "campos must have 3 elements")
    _check(background.numel() == 3, "background must have 3 elements")
    _check(softness > 0.0, "softness must be > 0")
    _check(image_width > 0 and image_height > 0, "invalid image dimensions")
    for t, n in zip(tensors, names):
        _check(t.dtype == torch.float32, f"{n} must be float32")
    if softnesses.numel() == 0:
        stride = 1
    elif softnesses.ndimension() == 1:
        _check(softnesses.numel() == P, "softnesses must have shape (P,), (P,3) or (0,)")
        stride = 1
    else:
        _check(softnesses.size(0) == P and softnesses.size(1) == 3,
               "softnesses must have shape (P,3)")
        stride = 3
    return P, stride


def _forward_core(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                  specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix,
                  campos, background, image_width, image_height, tan_fovx, tan_fovy, softness,
                  scale_modifier, color_model, view_model, use_view_grads, prefilter_edge_on,
                  conservative_bounds, debug, *, return_contrib=False, return_overdraw=False,
                  return_overdraw_hits=False, return_surface=False, overdraw_base_count=-1,
                  owner=False, return_median_depth=False, save=False, save_surface=False,
                  count_contrib=False, records=True, render=True):
    """rasterize_hexels3d_forward_impl (hexels3d_forward.cu:2679-3481).
    With `records` the per-surfel staged records are written once after the
    preprocess (hx_hexels3d_surfel_records) and the compositing stages them
    with asynchronous copies; they are returned for the backward.  With
    `render` False it stops after the binning and returns the preprocess
    and binning buffers under "binning"."""
    W, H = int(image_width), int(image_height)
    P, stride = _checks(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                        specular_ks, specular_log_s, opacities, softnesses, viewmatrix,
                        projmatrix, campos, background, W, H, float(softness), int(color_model),
                        int(view_model), bool(use_view_grads))
    dev = means3d.device
    f32 = dict(dtype=torch.float32, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    need_normals = return_surface or view_model == 2
    radii = torch.empty((P,), **i32)
    tile_radii = torch.empty((P, 2), **i32)
    points_xy_image = torch.empty((P, 2), **f32)
    points_xy_center = torch.empty((P, 2), **f32) if prefilter_edge_on else torch.empty((0,), **f32)
    depths = torch.empty((P,), **f32)
    transMats = torch.empty((P, 9), **f32)
    tiles_touched = torch.empty((P,), **i32)
    opacities_out = torch.empty((P,), **f32)
    softnesses_out = torch.empty((P, 3) if stride == 3 else (P,), **f32)
    view_dirs = torch.empty((P, 3), **f32)
    normals = torch.empty((P, 3), **f32) if need_normals else torch.empty((0,), **f32)
    soft_in = softnesses if softnesses.numel() > 0 else None
    with torch.cuda.device(dev):
        s = stream(dev)
        lib.call("hx_hexels3d_preprocess", P, ptr(means3d), ptr(scales), float(scale_modifier),
                 ptr(rotations), ptr(opacities), ptr(soft_in), float(softness), stride,
                 ptr(viewmatrix), ptr(projmatrix), ptr(campos), W, H, int(bool(prefilter_edge_on)),
                 int(bool(conservative_bounds)), ptr(radii), ptr(tile_radii),
                 ptr(points_xy_image), ptr(points_xy_center) if prefilter_edge_on else None,
                 ptr(depths), ptr(transMats), ptr(tiles_touched), ptr(opacities_out),
                 ptr(softnesses_out), ptr(view_dirs), ptr(normals) if need_normals else None, s)
        _mark("preprocess")
        # surfels in depth order, intersection offsets in that order and their
        # total (the one 8-byte read-back of the step, as in the reference)
        order = torch.empty((P,), **i32)
        offsets = torch.empty((P,), **i32)
        total = torch.empty((1,), dtype=torch.int64, device=dev)
        ws = workspace(lib.query("hx_hexels3d_depth_order_workspace_bytes", P), dev)
        lib.call("hx_hexels3d_depth_order", P, ptr(depths), ptr(tiles_touched), ptr(order),
                 ptr(offsets), ptr(total), ptr(ws), ws.numel(), s)
        _mark("scan")
        num_rendered = int(total.item()) if P > 0 else 0
        _check(num_rendered <= 2**31 - 1, "number of rendered intersections overflows int32")
        tx, ty = (W + 15) // 16, (H + 15) // 16
        ranges = torch.empty((tx * ty, 2), **i32)
        values_sorted = torch.empty((num_rendered,), **i32)
        ws = workspace(lib.query("hx_hexels3d_bin_ordered_workspace_bytes", num_rendered), dev)
        lib.call("hx_hexels3d_bin_ordered", P, num_rendered, W, H, ptr(points_xy_image),
                 ptr(order), ptr(offsets), ptr(radii), ptr(tile_radii), None, None,
                 ptr(values_sorted), ptr(ranges), ptr(ws), ws.numel(), s)

        _mark("bin")
        if not render:
            return dict(num_rendered=num_rendered, normals=normals, radii=radii,
                        binning=dict(ranges=ranges, point_list=values_sorted,
                                     transMats=transMats, opacities=opacities_out,
                                     softnesses=softnesses_out, view_dirs=view_dirs,
                                     depths=depths))
        # the compositing kernel writes every pixel of these outputs
        out_color = torch.empty((kNumChannels, H, W), **f32)
        contrib = torch.zeros((P,), **f32) if return_contrib else torch.empty((0,), **f32)
        overdraw = torch.empty((H, W), **f32) if return_overdraw else torch.empty((0,), **f32)
        overdraw_hits = (torch.empty((H, W), **f32) if return_overdraw_hits
                         else torch.empty((0,), **f32))
        if return_surface:
            surf_depth = torch.empty((H, W), **f32)
            surf_alpha = torch.empty((H, W), **f32)
            surf_maps = torch.empty((kNumChannels + 1 + int(return_median_depth), H, W), **f32)
        else:
            surf_depth = surf_alpha = surf_maps = torch.empty((0,), **f32)
        # per pixel: blended pairs, pairs evaluated after the warps' box cull
        contrib_count = torch.empty((2, H, W), **i32) if count_contrib else None
        # per intersection: the 8x4 pixel blocks that may blend it (lets the
        # backward skip the list entries no pixel of its block blends)
        blend_mask = (torch.empty((max(num_rendered, 1),), dtype=torch.uint8, device=dev)
                      if save else None)
        final_T = torch.empty((H, W), **f32) if save else torch.empty((0,), **f32)
        last_index = torch.empty((H, W), **i32) if save else torch.empty((0,), **i32)
        surf_state = None
        if save_surface and return_surface:
            surf_state = (torch.empty((H, W), **f32), torch.empty((H, W), **i32),
                          torch.empty((H, W), **f32), torch.empty((H, W), **f32),
                          torch.empty((H, W), **i32))
        own = None
        if owner:
            own = (torch.empty((H, W), dtype=torch.int64, device=dev),
                   torch.empty((H, W), **f32), torch.empty((2, H, W), **f32),
                   torch.empty((H, W), **f32), torch.empty((H, W), **f32),
                   torch.empty((H, W), **f32))
        rec = None
        if records and num_rendered > 0:
            rec = torch.empty((P, 32), **f32)  # 128-byte records
            lib.call("hx_hexels3d_surfel_records", P, W, H, ptr(transMats), ptr(opacities_out),
                     ptr(softnesses_out), stride, ptr(colors),
                     ptr(color_grads) if color_model >= 1 else None,
                     ptr(view_grads) if use_view_grads else None, ptr(view_dirs),
                     ptr(normals) if return_surface else None,
                     ptr(points_xy_center) if prefilter_edge_on else None, int(color_model),
                     int(bool(use_view_grads)), int(bool(return_surface)), ptr(rec), s)
        # launched even with nothing binned: every pixel is then the background
        lib.call("hx_hexels3d_render_forward", P, num_rendered, ptr(ranges),
                 ptr(values_sorted), ptr(points_xy_center) if prefilter_edge_on else None,
                 W, H, ptr(colors), ptr(color_grads) if color_model >= 1 else None,
                 ptr(color_quads) if color_model >= 2 else None,
                 ptr(view_grads) if use_view_grads else None,
                 ptr(specular_ks) if view_model == 2 else None,
                 ptr(specular_log_s) if view_model == 2 else None, ptr(view_dirs),
                 ptr(transMats), ptr(opacities_out), ptr(softnesses_out), stride,
                 ptr(background), ptr(normals) if need_normals else None,
                 int(overdraw_base_count), int(color_model), int(view_model),
                 int(bool(use_view_grads)), int(bool(return_median_depth)),
                 ptr(out_color), ptr(contrib) if return_contrib else None,
                 ptr(overdraw) if return_overdraw else None,
                 ptr(overdraw_hits) if return_overdraw_hits else None,
                 ptr(surf_depth) if return_surface else None,
                 ptr(surf_alpha) if return_surface else None,
                 ptr(surf_maps) if return_surface else None,
                 *(ptr(t) for t in own) if own else (None,) * 6,
                 ptr(final_T) if save else None, ptr(last_index) if save else None,
                 *(ptr(t) for t in surf_state) if surf_state else (None,) * 5,
                 ptr(contrib_count) if count_contrib else None, ptr(blend_mask), ptr(rec), s)
        _mark("render_fwd")
        if debug:
            torch.cuda.synchronize(dev)
    saved = None
    if save:
        saved = [radii, transMats, opacities_out, softnesses_out, view_dirs,
                 normals if view_model == 2 else torch.empty((0,), **f32),
                 points_xy_center, ranges, values_sorted, final_T, last_index]
    return dict(out_color=out_color, radii=radii, contrib=contrib, overdraw=overdraw,
                overdraw_hits=overdraw_hits, surf_depth=surf_depth, surf_alpha=surf_alpha,
                surf_maps=surf_maps, saved=saved, surf_state=surf_state, normals=normals,
                owner=own, num_rendered=num_rendered, contrib_count=contrib_count,
                blend_mask=blend_mask, records=rec)


def _forward_views_core(means3d, scales, rotations, colors, color_grads, view_grads, opacities,
                        cams, background, softness, color_model=1, view_model=1,
                        use_view_grads=True):
    """The RGB forward of a group of views of one scene (the training path:
    flat or linear colour, no or linear view model, one softness), binned
    together: one preprocess per view into view-major (V, P) buffers, one
    depth order and one binning of all the views' intersections
    (hx_hexels3d_depth_order_views / hx_hexels3d_bin_views, one 8-byte
    read-back for the group), then per view the staged records and the
    compositing.  Each view's lists are the ones _forward_core gives it.
    Returns one dict per view with out_color, radii, saved (the eleven
    buffers _backward_core takes: that view's slices, its ranges as offsets
    into the group's point_list), blend_mask (the group's, shared) and
    records."""
    e = _empty(means3d)
    V = len(cams)
    _check(V >= 1, "at least one view")
    _check(int(color_model) in (0, 1) and int(view_model) in (0, 1),
           "grouped views take the flat/linear colour and no/linear view models")
    W, H = int(cams[0].width), int(cams[0].height)
    _check(all(int(c.width) == W and int(c.height) == H for c in cams),
           "grouped views share one image size")
    P, stride = _checks(means3d, scales, rotations, colors, color_grads, e, view_grads, e, e,
                        opacities, e, cams[0].viewmatrix, cams[0].projmatrix, cams[0].campos,
                        background, W, H, float(softness), int(color_model), int(view_model),
                        bool(use_view_grads))
    dev = means3d.device
    f32 = dict(dtype=torch.float32, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    radii = torch.empty((V, P), **i32)
    tile_radii = torch.empty((V, P, 2), **i32)
    xy = torch.empty((V, P, 2), **f32)
    depths = torch.empty((V, P), **f32)
    transMats = torch.empty((V, P, 9), **f32)
    touched = torch.empty((V, P), **i32)
    op_out = torch.empty((V, P), **f32)
    soft_out = torch.empty((V, P), **f32)
    view_dirs = torch.empty((V, P, 3), **f32)
    tx, ty = (W + 15) // 16, (H + 15) // 16
    T = tx * ty
    outs = []
    with torch.cuda.device(dev):
        st = stream(dev)
        for v, cam in enumerate(cams):
            lib.call("hx_hexels3d_preprocess", P, ptr(means3d), ptr(scales), 1.0, ptr(rotations),
                     ptr(opacities), None, float(softness), stride, ptr(cam.viewmatrix),
                     ptr(cam.projmatrix), ptr(cam.campos), W, H, 0, 0, ptr(radii[v]),
                     ptr(tile_radii[v]), ptr(xy[v]), None, ptr(depths[v]), ptr(transMats[v]),
                     ptr(touched[v]), ptr(op_out[v]), ptr(soft_out[v]), ptr(view_dirs[v]), None,
                     st)
        order = torch.empty((V * P,), **i32)
        offsets = torch.empty((V * P,), **i32)
        total = torch.empty((1,), dtype=torch.int64, device=dev)
        ws = workspace(lib.query("hx_hexels3d_depth_order_views_workspace_bytes", V, P), dev)
        lib.call("hx_hexels3d_depth_order_views", V, P, ptr(depths), ptr(touched), ptr(order),
                 ptr(offsets), ptr(total), ptr(ws), ws.numel(), st)
        n = int(total.item()) if P > 0 else 0
        _check(n <= 2**31 - 1, "number of rendered intersections overflows int32")
        ranges = torch.empty((V, T, 2), **i32)
        point_list = torch.empty((n,), **i32)
        ws = workspace(lib.query("hx_hexels3d_bin_views_workspace_bytes", n), dev)
        lib.call("hx_hexels3d_bin_views", V, P, n, W, H, ptr(xy), ptr(order), ptr(offsets),
                 ptr(radii), ptr(tile_radii), ptr(point_list), ptr(ranges), ptr(ws), ws.numel(),
                 st)
        blend_mask = torch.empty((max(n, 1),), dtype=torch.uint8, device=dev)
        rec = torch.empty((V, P, 32), **f32) if n > 0 else None
        for v, cam in enumerate(cams):
            if rec is not None:
                lib.call("hx_hexels3d_surfel_records", P, W, H, ptr(transMats[v]), ptr(op_out[v]),
                         ptr(soft_out[v]), stride, ptr(colors),
                         ptr(color_grads) if color_model >= 1 else None,
                         ptr(view_grads) if use_view_grads else None, ptr(view_dirs[v]), None,
                         None, int(color_model), int(bool(use_view_grads)), 0, ptr(rec[v]), st)
            out_color = torch.empty((kNumChannels, H, W), **f32)
            final_T = torch.empty((H, W), **f32)
            last_index = torch.empty((H, W), **i32)
            lib.call("hx_hexels3d_render_forward", P, n, ptr(ranges[v]), ptr(point_list), None,
                     W, H, ptr(colors), ptr(color_grads) if color_model >= 1 else None, None,
                     ptr(view_grads) if use_view_grads else None, None, None, ptr(view_dirs[v]),
                     ptr(transMats[v]), ptr(op_out[v]), ptr(soft_out[v]), stride,
                     ptr(background), None, -1, int(color_model), int(view_model),
                     int(bool(use_view_grads)), 0, ptr(out_color), None, None, None, None, None,
                     None, *(None,) * 6, ptr(final_T), ptr(last_index), *(None,) * 5, None,
                     ptr(blend_mask), ptr(rec[v]) if rec is not None else None, st)
            saved = [radii[v], transMats[v], op_out[v], soft_out[v], view_dirs[v], _empty(xy),
                     _empty(xy), ranges[v], point_list, final_T, last_index]
            outs.append(dict(out_color=out_color, radii=radii[v], saved=saved,
                             blend_mask=blend_mask,
                             records=rec[v] if rec is not None else None, num_rendered=n))
    return outs


def _backward_core(means3d, means2d, scales, rotations, colors, color_grads, color_quads,
                   view_grads, specular_ks, specular_log_s, opacities, softnesses, viewmatrix,
                   projmatrix, campos, background, grad_out_color, grad_out_overdraw,
                   grad_out_surf_depth, grad_out_surf_alpha, grad_out_surf_normals, image_width,
                   image_height, tan_fovx, tan_fovy, softness, scale_modifier, color_model,
                   view_model, use_view_grads, overdraw_base_count, prefilter_edge_on,
                   conservative_bounds, debug, saved, surf_state=None, surf_normals=None,
                   accumulate_into=None, blend_mask=None, records=None):
    """rasterize_hexels3d_backward_impl (hexels3d_forward.cu:4882-5582) on the
    forward's saved state.  With `accumulate_into` (a dict from parameter
    name -- means3d, scales, rotations, colors, color_grads, view_grads,
    opacities -- to float32 buffers of the parameters' shapes) those gradients
    are added into the given buffers instead of returned fresh: gradient
    accumulation over views without a separate pass.  `blend_mask` is the
    forward's per-intersection mask of the same binning (or None)."""
    W, H = int(image_width), int(image_height)
    P, stride = _checks(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                        specular_ks, specular_log_s, opacities, softnesses, viewmatrix,
                        projmatrix, campos, background, W, H, float(softness), int(color_model),
                        int(view_model), bool(use_view_grads))
    for t, n in ((means2d, "means2d"), (grad_out_color, "grad_out_color"),
                 (grad_out_overdraw, "grad_out_overdraw"),
                 (grad_out_surf_depth, "grad_out_surf_depth"),
                 (grad_out_surf_alpha, "grad_out_surf_alpha"),
                 (grad_out_surf_normals, "grad_out_surf_normals")):
        check_input(t, n)
        _check(t.dtype == torch.float32, f"{n} must be float32")
    _check(means2d.numel() == 0 or (means2d.ndimension() == 2 and means2d.size(0) == P and
                                    means2d.size(1) in (3, 4)),
           "means2d must have shape (P,3), (P,4) or be empty")
    _check(grad_out_color.ndimension() == 3 and grad_out_color.size(0) == 3 and
           grad_out_color.size(1) == H and grad_out_color.size(2) == W,
           "grad_out_color must have shape (3,H,W)")
    for t, n in ((grad_out_overdraw, "grad_out_overdraw"),
                 (grad_out_surf_depth, "grad_out_surf_depth"),
                 (grad_out_surf_alpha, "grad_out_surf_alpha")):
        _check(t.numel() == 0 or tuple(t.shape) == (H, W), f"{n} must have shape (H,W) or be empty")
    _check(grad_out_surf_normals.numel() == 0 or (
        grad_out_surf_normals.ndimension() == 3 and grad_out_surf_normals.size(0) in (4, 5) and
        grad_out_surf_normals.size(1) == H and grad_out_surf_normals.size(2) == W),
        "grad_out_surf_normals must have shape (4,H,W), (5,H,W) or be empty")
    dev = means3d.device
    f32 = dict(dtype=torch.float32, device=dev)
    (radii, transMats, opacities_out, softnesses_out, view_dirs, normals_saved, points_xy_center,
     ranges, values_sorted, final_T, last_index) = saved
    num_rendered = values_sorted.numel()
    if records is not None:
        check_input(records, "records")
        _check(records.dtype == torch.float32 and tuple(records.shape) == (P, 32),
               "records must be the forward's (P, 32) float32 staged records")
    if blend_mask is not None:
        check_input(blend_mask, "blend_mask")
        _check(blend_mask.dtype == torch.uint8 and blend_mask.numel() >= num_rendered,
               "blend_mask must be uint8 with one entry per intersection")
    stride2d = means2d.size(1) if means2d.numel() > 0 else 3
    has_surface = (grad_out_surf_depth.numel() > 0 or grad_out_surf_alpha.numel() > 0 or
                   grad_out_surf_normals.numel() > 0)
    need_normals = view_model == 2 or grad_out_surf_normals.numel() > 0
    normals = surf_normals if (surf_normals is not None and surf_normals.numel() > 0) \
        else normals_saved
    _check(not need_normals or normals.numel() == 3 * P, "normals are required by this backward")
    acc = dict(accumulate_into or {})
    shapes = {"means3d": (P, 3), "means2d": tuple(means2d.shape), "scales": (P, 2),
              "rotations": (P, 4), "colors": (P, 3), "color_grads": tuple(color_grads.shape),
              "color_quads": tuple(color_quads.shape), "view_grads": tuple(view_grads.shape),
              "specular_ks": tuple(specular_ks.shape),
              "specular_log_s": tuple(specular_log_s.shape), "opacities": (P,),
              "softnesses": tuple(softnesses.shape), "normals": (P, 3) if need_normals else (0,),
              "transMats": (P, 9), "view_dirs": (P, 3),
              "center": (P, 2) if prefilter_edge_on else (0,)}
    for k, t in acc.items():
        _check(k in ("means3d", "scales", "rotations", "colors", "color_grads", "view_grads",
                     "opacities"), f"cannot accumulate the gradient of {k}")
        check_input(t, k)
        _check(t.dtype == torch.float32 and tuple(t.shape) == shapes[k],
               f"accumulation buffer {k} must be float32 of shape {shapes[k]}")
        _check(t.device == dev, f"accumulation buffer {k} must be on {dev}")
        # the geometry backward reads and writes rotations as float4 and
        # scales as float2
        align = {"rotations": 16, "scales": 8}.get(k, 4)
        _check(t.data_ptr() % align == 0,
               f"accumulation buffer {k} must start on a {align}-byte boundary")
    fresh = [k for k in shapes if k not in acc]
    g = dict(zip(fresh, _zero_views(dev, [shapes[k] for k in fresh])))
    g.update(acc)
    grad_means3d, grad_means2d, grad_scales, grad_rotations = (
        g["means3d"], g["means2d"], g["scales"], g["rotations"])
    grad_colors, grad_color_grads, grad_color_quads, grad_view_grads = (
        g["colors"], g["color_grads"], g["color_quads"], g["view_grads"])
    grad_specular_ks, grad_specular_log_s, grad_opacities, grad_softnesses = (
        g["specular_ks"], g["specular_log_s"], g["opacities"], g["softnesses"])
    grad_normals = g["normals"] if need_normals else None
    grad_transMats, grad_view_dirs = g["transMats"], g["view_dirs"]
    grad_center = g["center"] if prefilter_edge_on else None
    geo_acc = int(bool(acc))
    _check(not acc or all(k in acc for k in ("means3d", "scales", "rotations")),
           "accumulation needs means3d, scales and rotations buffers together")
    _check(not has_surface or surf_state is not None,
           "surface gradients need a forward run with surface outputs")
    nz = lambda t: ptr(t) if t.numel() > 0 else None  # noqa: E731
    with torch.cuda.device(dev):
        s = stream(dev)
        if num_rendered > 0:
            lib.call("hx_hexels3d_render_backward", P, num_rendered, ptr(ranges),
                     ptr(values_sorted), ptr(points_xy_center) if prefilter_edge_on else None,
                     ptr(grad_center), W, H, ptr(colors),
                     ptr(color_grads) if color_model >= 1 else None,
                     ptr(color_quads) if color_model >= 2 else None,
                     ptr(view_grads) if use_view_grads else None,
                     ptr(specular_ks) if view_model == 2 else None,
                     ptr(specular_log_s) if view_model == 2 else None, int(view_model),
                     ptr(view_dirs), ptr(transMats), ptr(opacities_out), ptr(softnesses_out),
                     stride, ptr(background), ptr(grad_out_color), nz(grad_out_overdraw),
                     nz(grad_out_surf_depth) if has_surface else None,
                     nz(grad_out_surf_alpha) if has_surface else None,
                     nz(grad_out_surf_normals) if has_surface else None,
                     int(has_surface and grad_out_surf_normals.numel() > 0 and
                         grad_out_surf_normals.size(0) == 5),
                     ptr(normals) if need_normals else None, ptr(grad_colors),
                     ptr(grad_color_grads) if color_model >= 1 else None,
                     ptr(grad_color_quads) if color_model >= 2 else None,
                     ptr(grad_view_grads) if use_view_grads else None,
                     ptr(grad_specular_ks) if view_model == 2 else None,
                     ptr(grad_specular_log_s) if view_model == 2 else None,
                     ptr(grad_opacities),
                     ptr(grad_softnesses) if softnesses.numel() > 0 else None,
                     ptr(grad_transMats), ptr(grad_means2d) if stride2d == 4 and
                     means2d.numel() > 0 else None, ptr(grad_view_dirs), ptr(grad_normals),
                     int(overdraw_base_count), int(color_model), int(bool(use_view_grads)),
                     ptr(final_T), ptr(last_index),
                     *(ptr(t) for t in surf_state) if has_surface else (None,) * 5,
                     ptr(blend_mask), ptr(records), s)
            _mark("render_bwd")
            lib.call("hx_hexels3d_geometry_backward", P, num_rendered, ptr(means3d), ptr(scales),
                     float(scale_modifier), ptr(rotations), ptr(projmatrix), ptr(campos), W, H,
                     ptr(radii), ptr(transMats), ptr(grad_transMats), ptr(grad_view_dirs),
                     ptr(grad_normals), ptr(grad_center), ptr(grad_means3d),
                     ptr(grad_means2d) if means2d.numel() > 0 else None, int(stride2d),
                     ptr(grad_scales), ptr(grad_rotations), geo_acc, s)
            _mark("geometry_bwd")
        if debug:
            torch.cuda.synchronize(dev)
    return (grad_means3d, grad_means2d, grad_scales, grad_rotations, grad_colors,
            grad_color_grads, grad_color_quads, grad_view_grads, grad_specular_ks,
            grad_specular_log_s, grad_opacities, grad_softnesses)


# ---------------------------------------------------------------------------
# the reference's entry points (ext.cpp:6-22)
# ---------------------------------------------------------------------------
def rasterize_hexels3d_forward(*args):
    o = _forward_core(*args)
    return o["out_color"], o["radii"]


def rasterize_hexels3d_forward_cached(*args):
    o = _forward_core(*args, save=True)
    return o["out_color"], o["radii"], o["saved"]


def rasterize_hexels3d_owner_forward(*args):
    o = _forward_core(*args, owner=True)
    return (o["out_color"], o["radii"], *o["owner"])


def rasterize_hexels3d_forward_with_contrib(*args):
    o = _forward_core(*args, return_contrib=True)
    return o["out_color"], o["radii"], o["contrib"]


def _split_overdraw(args):
    # (..., use_view_grads, overdraw_base_count, prefilter, conservative, debug)
    base = list(args[:24])
    odb, pre, cons, dbg = args[24:28]
    return base + [pre, cons, dbg], int(odb)


def rasterize_hexels3d_forward_with_overdraw(*args):
    a, odb = _split_overdraw(args)
    o = _forward_core(*a, return_overdraw=True, overdraw_base_count=odb)
    return o["out_color"], o["radii"], o["overdraw"]


def rasterize_hexels3d_forward_with_contrib_overdraw(*args):
    a, odb = _split_overdraw(args)
    o = _forward_core(*a, return_contrib=True, return_overdraw=True, overdraw_base_count=odb)
    return o["out_color"], o["radii"], o["contrib"], o["overdraw"]


def rasterize_hexels3d_forward_with_overdraw_hits(*args):
    a, odb = _split_overdraw(args)
    o = _forward_core(*a, return_overdraw=True, return_overdraw_hits=True,
                      overdraw_base_count=odb)
    return o["out_color"], o["radii"], o["overdraw"], o["overdraw_hits"]


def rasterize_hexels3d_forward_with_contrib_overdraw_hits(*args):
    a, odb = _split_overdraw(args)
    o = _forward_core(*a, return_contrib=True, return_overdraw=True, return_overdraw_hits=True,
                      overdraw_base_count=odb)
    return o["out_color"], o["radii"], o["contrib"], o["overdraw"], o["overdraw_hits"]


def _all(args, median: bool):
    base = list(args[:24])
    (ret_contrib, ret_overdraw, ret_hits, ret_surface, odb, pre, cons, dbg) = args[24:32]
    o = _forward_core(*base, pre, cons, dbg, return_contrib=bool(ret_contrib),
                      return_overdraw=bool(ret_overdraw), return_overdraw_hits=bool(ret_hits),
                      return_surface=bool(ret_surface), overdraw_base_count=int(odb),
                      return_median_depth=median)
    return (o["out_color"], o["radii"], o["contrib"], o["overdraw"], o["overdraw_hits"],
            o["surf_depth"], o["surf_alpha"], o["surf_maps"])


def rasterize_hexels3d_forward_all(*args):
    return _all(args, False)


def rasterize_hexels3d_forward_median(*args):
    return _all(args, True)


def rasterize_hexels3d_backward_cached(*args):
    if len(args) != 35:
        raise TypeError("rasterize_hexels3d_backward_cached takes 35 arguments")
    saved = list(args[34])
    _check(len(saved) == 11, "Expected eleven saved rasterizer buffers")
    for t in saved:
        check_input(t, "saved")
    gs = args[17:21]
    _check(all(t.numel() == 0 for t in gs),
           "Cached RGB backward does not accept auxiliary gradients")
    return _backward_core(*args[:34], saved)


def rasterize_hexels3d_backward(*args):
    """Uncached backward: re-runs the forward (preprocess, binning and, for
    surface gradients, the surface state) and then the cached backward."""
    if len(args) != 34:
        raise TypeError("rasterize_hexels3d_backward takes 34 arguments")
    (means3d, means2d, scales, rotations, colors, color_grads, color_quads, view_grads,
     specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix, campos,
     background, g_color, g_overdraw, g_depth, g_alpha, g_normals, W, H, tfx, tfy, softness,
     mod, cm, vm, uvg, odb, pre, cons, dbg) = args
    surface = g_depth.numel() > 0 or g_alpha.numel() > 0 or g_normals.numel() > 0
    median = surface and g_normals.numel() > 0 and g_normals.size(0) == 5
    o = _forward_core(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                      specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix,
                      campos, background, W, H, tfx, tfy, softness, mod, cm, vm, uvg, pre, cons,
                      False, return_surface=surface, overdraw_base_count=odb,
                      return_median_depth=median, save=True, save_surface=surface)
    return _backward_core(*args, o["saved"], surf_state=o["surf_state"],
                          surf_normals=o["normals"] if surface else None,
                          blend_mask=o["blend_mask"], records=o["records"])


def _exact_core(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix,
                campos, background, native_image, selected_mask, pixel_mask, W, H, softness,
                scale_modifier, color_model, view_model, use_view_grads, exact_mode, crop,
                compute_risk, debug):
    """rasterize_hexels3d_exact_sort_forward_impl (hexels3d_forward.cu:4217-4721):
    preprocess and binning as the forward, then each enabled crop pixel's
    hits re-sorted by depth and composited in that order."""
    W, H = int(W), int(H)
    P, stride = _checks(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                        specular_ks, specular_log_s, opacities, softnesses, viewmatrix,
                        projmatrix, campos, background, W, H, float(softness), int(color_model),
                        int(view_model), bool(use_view_grads))
    for t, n in ((native_image, "native_image"), (selected_mask, "selected_mask"),
                 (pixel_mask, "pixel_mask")):
        check_input(t, n)
    dev = means3d.device
    for t in (native_image, selected_mask, pixel_mask):
        _check(t.device == dev, "all exact-sort tensors must be on the same CUDA device")
    _check(selected_mask.dtype == torch.bool, "selected_mask must be bool")
    _check(pixel_mask.dtype == torch.bool, "pixel_mask must be bool")
    mode = int(exact_mode)
    if mode == 5:
        _check(selected_mask.numel() == 0, "selected_mask must be empty in pixel-mask mode")
        _check(tuple(pixel_mask.shape) == (H, W), "pixel_mask must have shape (H,W)")
    else:
        _check(selected_mask.ndimension() == 1 and selected_mask.numel() == P,
               "selected_mask must have shape (P,)")
        _check(pixel_mask.numel() == 0, "pixel_mask must be empty outside pixel-mask mode")
    _check(tuple(native_image.shape) == (3, H, W) and native_image.dtype == torch.float32,
           "native_image must have shape (3,H,W)")
    _check(W * H <= 2**32 - 1, "image has too many pixels for exact-sort keys")
    _check(0 <= mode <= 5, "invalid exact sort mode")
    x0, y0, x1, y1 = (int(c) for c in crop)
    _check(0 <= x0 < x1 <= W and 0 <= y0 < y1 <= H,
           "crop must satisfy 0 <= x0 < x1 <= W and 0 <= y0 < y1 <= H")
    e = _empty(means3d)
    o = _forward_core(means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
                      specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix,
                      campos, background, W, H, 1.0, 1.0, softness, scale_modifier, color_model,
                      view_model, use_view_grads, False, False, False, records=False,
                      render=False)
    b = o["binning"]
    n = o["num_rendered"]
    i32 = dict(dtype=torch.int32, device=dev)
    out_color = native_image.clone()
    order_changed = torch.zeros((H, W), dtype=torch.bool, device=dev)
    hit_counts = torch.zeros((H, W), **i32)
    enabled = torch.zeros((H, W), dtype=torch.bool, device=dev)
    risk = torch.zeros((H, W), dtype=torch.float32, device=dev)
    record_counts = torch.zeros((H * W,), **i32)
    cm, vm, uvg = int(color_model), int(view_model), bool(use_view_grads)
    common = (P, n, ptr(b["ranges"]), ptr(b["point_list"]) if n > 0 else None, W, H,
              ptr(colors), ptr(color_grads) if cm >= 1 else None,
              ptr(color_quads) if cm >= 2 else None, ptr(view_grads) if uvg else None,
              ptr(specular_ks) if vm == 2 else None, ptr(specular_log_s) if vm == 2 else None,
              ptr(b["view_dirs"]), ptr(o["normals"]) if vm == 2 else None, ptr(b["transMats"]),
              ptr(b["opacities"]), ptr(b["softnesses"]), stride, ptr(background),
              ptr(b["depths"]), ptr(selected_mask) if selected_mask.numel() else None,
              ptr(pixel_mask) if pixel_mask.numel() else None, cm, vm, int(uvg), mode, x0, y0,
              x1, y1)
    with torch.cuda.device(dev):
        st = stream(dev)
        lib.call("hx_hexels3d_exact_count", *common, ptr(hit_counts), ptr(record_counts),
                 ptr(enabled), ptr(risk) if compute_risk else None, st)
        offsets = torch.empty((H * W,), **i32)
        total = torch.empty((1,), dtype=torch.int64, device=dev)
        ws = workspace(lib.query("hx_scan_workspace_bytes", H * W), dev)
        lib.call("hx_inclusive_scan_i32", ptr(record_counts), ptr(offsets), H * W, ptr(total),
                 ptr(ws), ws.numel(), st)
        num_records = int(total.item())
        _check(num_records <= 2**31 - 1,
               "exact-sort crop has too many hit records; use smaller crop strips")
        ws = workspace(lib.query("hx_hexels3d_exact_resolve_workspace_bytes", num_records), dev)
        lib.call("hx_hexels3d_exact_resolve", *common, ptr(enabled), ptr(record_counts),
                 ptr(offsets), num_records, ptr(out_color), ptr(order_changed), ptr(ws),
                 ws.numel(), st)
        if debug:
            torch.cuda.synchronize(dev)
    return out_color, order_changed, hit_counts, enabled, risk


def rasterize_hexels3d_exact_sort_forward(*args):
    """(out_color, order_changed, hit_counts, enabled_mask): the enabled crop
    pixels of native_image recomposited with their hits sorted by depth at
    the pixel (hexels3d_forward.cu:4722-4791)."""
    if len(args) != 30:
        raise TypeError("rasterize_hexels3d_exact_sort_forward takes 30 arguments")
    (m3, sc, rot, col, cg, cq, vg, ks, ls, op, soft, vm_, pm, cp, bg, native, selected, W, H,
     softness, mod, cm, vm, uvg, mode, x0, y0, x1, y1, dbg) = args
    pixel_mask = torch.empty((0,), dtype=torch.bool, device=selected.device)
    out = _exact_core(m3, sc, rot, col, cg, cq, vg, ks, ls, op, soft, vm_, pm, cp, bg, native,
                      selected, pixel_mask, W, H, softness, mod, cm, vm, uvg, mode,
                      (x0, y0, x1, y1), False, dbg)
    return out[0], out[1], out[2], out[3]


def rasterize_hexels3d_pixel_risk_forward(*args):
    """(out_color, risk_map, order_changed, hit_counts, enabled_mask): the
    pixel-mask exact sort plus the inversion risk of the list order over the
    crop (hexels3d_forward.cu:4793-4880)."""
    if len(args) != 29:
        raise TypeError("rasterize_hexels3d_pixel_risk_forward takes 29 arguments")
    (m3, sc, rot, col, cg, cq, vg, ks, ls, op, soft, vm_, pm, cp, bg, native, pixel_mask, W, H,
     softness, mod, cm, vm, uvg, x0, y0, x1, y1, dbg) = args
    selected = torch.empty((0,), dtype=torch.bool, device=pixel_mask.device)
    out = _exact_core(m3, sc, rot, col, cg, cq, vg, ks, ls, op, soft, vm_, pm, cp, bg, native,
                      selected, pixel_mask, W, H, softness, mod, cm, vm, uvg, 5,
                      (x0, y0, x1, y1), True, dbg)
    return out[0], out[4], out[1], out[2], out[3]


def _sig(name, n_tensor, n_total, returns):
    types = ["torch.Tensor"] * n_tensor + ["int", "int", "float", "float", "float", "float",
                                           "int", "int", "bool", "bool", "bool",
                                           "bool"][: n_total - n_tensor]
    params = ", ".join(f"arg{i}: {t}" for i, t in enumerate(types))
    return f"{name}({params}) -> tuple[{', '.join(['torch.Tensor'] * returns)}]\n"


# pybind-style signatures, so callers that validate the extension's arity by
# its docstrings (gsplat/cuda_hexels3d/__init__.py of the reference) accept it.
rasterize_hexels3d_forward.__doc__ = _sig("rasterize_hexels3d_forward", 15, 27, 2)
rasterize_hexels3d_backward.__doc__ = (
    "rasterize_hexels3d_backward("
    + ", ".join([f"arg{i}: torch.Tensor" for i in range(21)]
                + [f"arg{21 + i}: {t}" for i, t in enumerate(
                    ["int", "int", "float", "float", "float", "float", "int", "int", "bool",
                     "int", "bool", "bool", "bool"])])
    + ") -> tuple[" + ", ".join(["torch.Tensor"] * 12) + "]\n")
