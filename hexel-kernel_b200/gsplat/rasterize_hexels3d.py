"""3D hexel surfel rasterisation — same public API as the reference's
gsplat/rasterize_hexels3d.py (functions, keyword arguments, returns, errors).

One autograd Function serves every differentiable variant (RGB, contrib,
overdraw, surface outputs): its forward always keeps the binning and the
per-pixel compositing state the backward needs, so the backward never
re-runs preprocessing, binning or a forward walk (the reference re-runs all
three for its surface-output path, gsplat/rasterize_hexels3d.py:2294-2491 and
hexels3d_forward.cu:5209-5310).  Results are the same; only time and memory
traffic differ.
"""

from __future__ import annotations

from typing import Optional, Literal, Tuple

import torch
from torch import Tensor
from torch.autograd import Function

ColorModel = Literal["flat", "linear", "quadratic", "quadratic_bounded"]
ViewModel = Literal["none", "linear", "lobe"]

_COLOR_MODEL_TO_INT = {"flat": 0, "linear": 1, "quadratic": 2, "quadratic_bounded": 3}
_VIEW_MODEL_TO_INT = {"none": 0, "linear": 1, "lobe": 2}


def _color_model_to_int(color_model) -> int:
    if isinstance(color_model, int):
        if color_model in (0, 1, 2, 3):
            return int(color_model)
        raise ValueError(
            "color_model int must be one of: 0 (flat), 1 (linear), "
            "2 (quadratic), 3 (quadratic_bounded)"
        )
    if color_model not in _COLOR_MODEL_TO_INT:
        raise ValueError("color_model must be one of: flat, linear, quadratic, quadratic_bounded")
    return _COLOR_MODEL_TO_INT[color_model]


def _view_model_to_int(view_model) -> int:
    if isinstance(view_model, int):
        if view_model in (0, 1, 2):
            return int(view_model)
        raise ValueError("view_model int must be one of: 0 (none), 1 (linear), 2 (lobe)")
    if view_model not in _VIEW_MODEL_TO_INT:
        raise ValueError("view_model must be one of: none, linear, lobe")
    return _VIEW_MODEL_TO_INT[view_model]


def _empty_like(x: Tensor) -> Tensor:
    return torch.empty((0,), device=x.device, dtype=x.dtype)


def _prepare(means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s,
             softnesses, color_model, view_model, use_view_grads):
    """Normalises models and replaces unused appearance tensors by empty ones
    (reference gsplat/rasterize_hexels3d.py:60-78, 1091-1117)."""
    cm = _color_model_to_int(color_model)
    vm = _view_model_to_int(view_model)
    uvg = bool(use_view_grads) and vm == 1
    empty = _empty_like(means3d)
    cg = color_grads if cm >= 1 else empty
    if cm in (2, 3):
        if color_quads is None:
            raise ValueError("color_quads must be provided for a quadratic color model")
        cq = color_quads
    else:
        cq = empty
    vg = view_grads if uvg else empty
    ks, ls = empty, empty
    if vm == 2:
        if specular_ks is None or specular_log_s is None:
            raise ValueError("specular_ks and specular_log_s must be provided when view_model='lobe'")
        ks, ls = specular_ks, specular_log_s
    soft = softnesses.contiguous() if softnesses is not None else empty
    return cm, vm, uvg, cg.contiguous(), cq.contiguous(), vg.contiguous(), ks.contiguous(), \
        ls.contiguous(), soft


def _C():
    from .cuda_hexels3d import _C as C

    return C


# ---------------------------------------------------------------------------
# forward-only entry points (reference gsplat/rasterize_hexels3d.py:81-750)
# ---------------------------------------------------------------------------
def _fwd_args(means3d, scales, rotations, colors, color_grads, view_grads, opacities, viewmatrix,
              projmatrix, campos, background, image_width, image_height, tan_fovx, tan_fovy,
              softness, softnesses, color_quads, specular_ks, specular_log_s, scale_modifier,
              color_model, view_model, use_view_grads):
    cm, vm, uvg, cg, cq, vg, ks, ls, soft = _prepare(
        means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s, softnesses,
        color_model, view_model, use_view_grads)
    return (means3d.contiguous(), scales.contiguous(), rotations.contiguous(),
            colors.contiguous(), cg, cq, vg, ks, ls, opacities.contiguous(), soft,
            viewmatrix.contiguous(), projmatrix.contiguous(), campos.contiguous(),
            background.contiguous(), int(image_width), int(image_height), float(tan_fovx),
            float(tan_fovy), float(softness), float(scale_modifier), cm, vm, uvg)


def rasterize_hexels3d_forward(means3d, scales, rotations, colors, color_grads, view_grads,
                               opacities, viewmatrix, projmatrix, campos, background, image_width,
                               image_height, tan_fovx, tan_fovy, softness, softnesses=None, *,
                               color_quads=None, specular_ks=None, specular_log_s=None,
                               scale_modifier=1.0, color_model="linear", view_model="linear",
                               use_view_grads=True, prefilter_edge_on=False,
                               conservative_bounds=False, debug=False) -> Tuple[Tensor, Tensor]:
    """Inference render: (out_color (3,H,W), radii (P,))."""
    a = _fwd_args(means3d, scales, rotations, colors, color_grads, view_grads, opacities,
                  viewmatrix, projmatrix, campos, background, image_width, image_height,
                  tan_fovx, tan_fovy, softness, softnesses, color_quads, specular_ks,
                  specular_log_s, scale_modifier, color_model, view_model, use_view_grads)
    return _C().rasterize_hexels3d_forward(*a, bool(prefilter_edge_on),
                                           bool(conservative_bounds), bool(debug))


def rasterize_hexels3d_owner_forward(means3d, scales, rotations, colors, color_grads, view_grads,
                                     opacities, viewmatrix, projmatrix, campos, background,
                                     image_width, image_height, tan_fovx, tan_fovy, softness,
                                     softnesses=None, *, color_quads=None, specular_ks=None,
                                     specular_log_s=None, scale_modifier=1.0,
                                     color_model="linear", view_model="linear",
                                     use_view_grads=True, prefilter_edge_on=False,
                                     conservative_bounds=False, debug=False):
    """(out_color, radii, owner_id, owner_weight, owner_uv, owner_sdf,
    owner_depth, total_alpha): the surfel with the largest blending weight
    per pixel."""
    a = _fwd_args(means3d, scales, rotations, colors, color_grads, view_grads, opacities,
                  viewmatrix, projmatrix, campos, background, image_width, image_height,
                  tan_fovx, tan_fovy, softness, softnesses, color_quads, specular_ks,
                  specular_log_s, scale_modifier, color_model, view_model, use_view_grads)
    return _C().rasterize_hexels3d_owner_forward(*a, bool(prefilter_edge_on),
                                                 bool(conservative_bounds), bool(debug))


def _forward_variant(name, with_overdraw):
    def fn(means3d, scales, rotations, colors, color_grads, view_grads, opacities, viewmatrix,
           projmatrix, campos, background, image_width, image_height, tan_fovx, tan_fovy,
           softness, softnesses=None, *, color_quads=None, specular_ks=None,
           specular_log_s=None, scale_modifier=1.0, color_model="linear", view_model="linear",
           use_view_grads=True, overdraw_base_count=-1, prefilter_edge_on=False,
           conservative_bounds=False, debug=False):
        a = _fwd_args(means3d, scales, rotations, colors, color_grads, view_grads, opacities,
                      viewmatrix, projmatrix, campos, background, image_width, image_height,
                      tan_fovx, tan_fovy, softness, softnesses, color_quads, specular_ks,
                      specular_log_s, scale_modifier, color_model, view_model, use_view_grads)
        extra = (int(overdraw_base_count),) if with_overdraw else ()
        return getattr(_C(), name)(*a, *extra, bool(prefilter_edge_on),
                                   bool(conservative_bounds), bool(debug))

    fn.__name__ = name
    fn.__doc__ = f"Inference render with extra per-pixel / per-surfel outputs ({name})."
    return fn


rasterize_hexels3d_forward_with_contrib = _forward_variant(
    "rasterize_hexels3d_forward_with_contrib", False)
rasterize_hexels3d_forward_with_overdraw = _forward_variant(
    "rasterize_hexels3d_forward_with_overdraw", True)
rasterize_hexels3d_forward_with_overdraw_hits = _forward_variant(
    "rasterize_hexels3d_forward_with_overdraw_hits", True)
rasterize_hexels3d_forward_with_contrib_overdraw = _forward_variant(
    "rasterize_hexels3d_forward_with_contrib_overdraw", True)
rasterize_hexels3d_forward_with_contrib_overdraw_hits = _forward_variant(
    "rasterize_hexels3d_forward_with_contrib_overdraw_hits", True)


_EXACT_SORT_MODE_TO_INT = {"center_replay": 0, "hybrid": 1, "selected_all": 2, "crop_all": 3,
                          "boundary_tail": 4}


def _exact_inputs(means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s,
                  softnesses, color_model, view_model, use_view_grads, crop_xyxy, W, H,
                  prefilter_edge_on, what):
    if prefilter_edge_on:
        raise ValueError(f"The {what} oracle does not support prefilter_edge_on=True")
    if crop_xyxy is None:
        crop_xyxy = (0, 0, int(W), int(H))
    if len(crop_xyxy) != 4:
        raise ValueError("crop_xyxy must contain (x0, y0, x1, y1)")
    return _prepare(means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s,
                    softnesses, color_model, view_model, use_view_grads), tuple(crop_xyxy)


def rasterize_hexels3d_exact_sort_forward(means3d: Tensor, scales: Tensor, rotations: Tensor,
                                          colors: Tensor, color_grads: Tensor, view_grads: Tensor,
                                          opacities: Tensor, viewmatrix: Tensor,
                                          projmatrix: Tensor, campos: Tensor, background: Tensor,
                                          native_image: Tensor, selected_mask: Tensor,
                                          image_width: int, image_height: int, softness: float,
                                          softnesses: Optional[Tensor] = None, *,
                                          color_quads: Optional[Tensor] = None,
                                          specular_ks: Optional[Tensor] = None,
                                          specular_log_s: Optional[Tensor] = None,
                                          scale_modifier: float = 1.0, color_model="linear",
                                          view_model="linear", use_view_grads: bool = True,
                                          mode: str = "center_replay", crop_xyxy=None,
                                          prefilter_edge_on: bool = False, debug: bool = False):
    """Diagnostic replay of a crop with each enabled pixel's hits re-sorted
    by the depth at the pixel (reference gsplat/rasterize_hexels3d.py:750-852):
    returns (image, order_changed, hit_counts, enabled_mask); pixels outside
    the crop or not enabled keep native_image.  selected_mask (P,) bool marks
    the surfels whose pixels are replayed in the hybrid and selected modes."""
    if mode not in _EXACT_SORT_MODE_TO_INT:
        raise ValueError(f"Unknown exact-sort mode: {mode}")
    (cm, vm, uvg, cg, cq, vg, ks, ls, soft), crop = _exact_inputs(
        means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s, softnesses,
        color_model, view_model, use_view_grads, crop_xyxy, image_width, image_height,
        prefilter_edge_on, "exact-sort")
    return _C().rasterize_hexels3d_exact_sort_forward(
        means3d.contiguous(), scales.contiguous(), rotations.contiguous(), colors.contiguous(),
        cg, cq, vg, ks, ls, opacities.contiguous(), soft, viewmatrix.contiguous(),
        projmatrix.contiguous(), campos.contiguous(), background.contiguous(),
        native_image.contiguous(), selected_mask.contiguous(), int(image_width),
        int(image_height), float(softness), float(scale_modifier), cm, vm, uvg,
        _EXACT_SORT_MODE_TO_INT[mode], *(int(c) for c in crop), bool(debug))


def rasterize_hexels3d_pixel_risk_forward(means3d: Tensor, scales: Tensor, rotations: Tensor,
                                          colors: Tensor, color_grads: Tensor, view_grads: Tensor,
                                          opacities: Tensor, viewmatrix: Tensor,
                                          projmatrix: Tensor, campos: Tensor, background: Tensor,
                                          native_image: Tensor, pixel_mask: Tensor,
                                          image_width: int, image_height: int, softness: float,
                                          softnesses: Optional[Tensor] = None, *,
                                          color_quads: Optional[Tensor] = None,
                                          specular_ks: Optional[Tensor] = None,
                                          specular_log_s: Optional[Tensor] = None,
                                          scale_modifier: float = 1.0, color_model="linear",
                                          view_model="linear", use_view_grads: bool = True,
                                          crop_xyxy=None, prefilter_edge_on: bool = False,
                                          debug: bool = False):
    """Diagnostic inversion-risk map of the compositing order over a crop,
    plus the exact depth re-sort of the pixels in pixel_mask (H,W) bool
    (reference gsplat/rasterize_hexels3d.py:854-955): returns (image, risk,
    order_changed, hit_counts, enabled_mask)."""
    (cm, vm, uvg, cg, cq, vg, ks, ls, soft), crop = _exact_inputs(
        means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s, softnesses,
        color_model, view_model, use_view_grads, crop_xyxy, image_width, image_height,
        prefilter_edge_on, "pixel-risk")
    return _C().rasterize_hexels3d_pixel_risk_forward(
        means3d.contiguous(), scales.contiguous(), rotations.contiguous(), colors.contiguous(),
        cg, cq, vg, ks, ls, opacities.contiguous(), soft, viewmatrix.contiguous(),
        projmatrix.contiguous(), campos.contiguous(), background.contiguous(),
        native_image.contiguous(), pixel_mask.contiguous(), int(image_width),
        int(image_height), float(softness), float(scale_modifier), cm, vm, uvg,
        *(int(c) for c in crop), bool(debug))


# ---------------------------------------------------------------------------
# differentiable rendering
# ---------------------------------------------------------------------------
class _RasterizeHexels3D(Function):
    """Differentiable render of every output variant; keeps the forward's
    binning and per-pixel state for the backward."""

    @staticmethod
    def forward(ctx, means3d, means2d, scales, rotations, colors, color_grads, color_quads,
                view_grads, specular_ks, specular_log_s, opacities, softnesses, viewmatrix,
                projmatrix, campos, background, opts: dict):
        C = _C()
        o = C._forward_core(
            means3d, scales, rotations, colors, color_grads, color_quads, view_grads,
            specular_ks, specular_log_s, opacities, softnesses, viewmatrix, projmatrix, campos,
            background, opts["image_width"], opts["image_height"], opts["tan_fovx"],
            opts["tan_fovy"], opts["softness"], opts["scale_modifier"], opts["color_model"],
            opts["view_model"], opts["use_view_grads"], opts["prefilter_edge_on"],
            opts["conservative_bounds"], opts["debug"],
            return_contrib=opts["return_contrib"], return_overdraw=opts["return_overdraw"],
            return_overdraw_hits=opts["return_overdraw_hits"],
            return_surface=opts["return_surface"],
            overdraw_base_count=opts["overdraw_base_count"],
            return_median_depth=opts["return_median_depth"], save=True,
            save_surface=opts["return_surface"])
        saved = o["saved"]
        surf = list(o["surf_state"]) if o["surf_state"] is not None else []
        ctx.n_surf = len(surf)
        ctx.save_for_backward(means3d, means2d, scales, rotations, colors, color_grads,
                              color_quads, view_grads, specular_ks, specular_log_s, opacities,
                              softnesses, viewmatrix, projmatrix, campos, background, *saved,
                              *surf, o["normals"], o["blend_mask"], o["records"])
        ctx.opts = opts
        ctx.mark_non_differentiable(o["radii"], o["contrib"], o["overdraw_hits"])
        return (o["out_color"], o["radii"], o["contrib"], o["overdraw"], o["overdraw_hits"],
                o["surf_depth"], o["surf_alpha"], o["surf_maps"])

    @staticmethod
    def backward(ctx, g_color, g_radii, g_contrib, g_overdraw, g_hits, g_depth, g_alpha, g_maps):
        t = ctx.saved_tensors
        inputs, saved = t[:16], list(t[16:27])
        surf = t[27:27 + ctx.n_surf]
        normals = t[27 + ctx.n_surf]
        blend_mask = t[28 + ctx.n_surf]
        records = t[29 + ctx.n_surf]
        opts = ctx.opts
        empty = _empty_like(inputs[0])

        def grad_or_empty(g, enabled):
            if not enabled or g is None:
                return empty
            return g.contiguous()

        go = grad_or_empty(g_overdraw, opts["return_overdraw"])
        gd = grad_or_empty(g_depth, opts["return_surface"])
        ga = grad_or_empty(g_alpha, opts["return_surface"])
        gm = grad_or_empty(g_maps, opts["return_surface"])
        grads = _C()._backward_core(
            *inputs, g_color.contiguous(), go, gd, ga, gm, opts["image_width"],
            opts["image_height"], opts["tan_fovx"], opts["tan_fovy"], opts["softness"],
            opts["scale_modifier"], opts["color_model"], opts["view_model"],
            opts["use_view_grads"], opts["overdraw_base_count"], opts["prefilter_edge_on"],
            opts["conservative_bounds"], opts["debug"], saved,
            surf_state=tuple(surf) if surf else None,
            surf_normals=normals if opts["return_surface"] else None, blend_mask=blend_mask,
            records=records)
        means2d = inputs[1]
        g2d = grads[1] if means2d.numel() > 0 else None
        return (grads[0], g2d, *grads[2:], None, None, None, None, None)


def rasterize_hexels3d(
    means3d: Tensor, scales: Tensor, rotations: Tensor, colors: Tensor, color_grads: Tensor,
    view_grads: Tensor, opacities: Tensor, viewmatrix: Tensor, projmatrix: Tensor,
    campos: Tensor, background: Tensor, image_width: int, image_height: int, tan_fovx: float,
    tan_fovy: float, softness: float, softnesses: Tensor | None = None, *,
    means2d: Tensor | None = None, color_quads: Tensor | None = None,
    specular_ks: Tensor | None = None, specular_log_s: Tensor | None = None,
    scale_modifier: float = 1.0, color_model: ColorModel | int = "linear",
    view_model: ViewModel | int = "linear", use_view_grads: bool = True,
    return_contrib: bool = False, return_overdraw: bool = False,
    return_overdraw_hits: bool = False, return_surface: bool = False,
    return_distortion: bool = False, return_median_depth: bool = False,
    overdraw_base_count: int = -1, prefilter_edge_on: bool = False,
    conservative_bounds: bool = False, debug: bool = False,
) -> Tuple[Tensor, ...]:
    """Differentiable render of 3D hexel surfels (WXYZ quaternions, 2D tangent
    scales) with front-to-back alpha compositing.

    Returns (out_color (3,H,W), radii (P,)) followed, as requested, by contrib
    (P,), overdraw (H,W), overdraw_hits (H,W), and with return_surface depth
    (H,W), alpha (H,W), normals (3,H,W), [distortion (H,W)], [median (H,W)].
    ``means2d`` (P,3) or (P,4) is a screen-gradient proxy, not a position
    input: its .grad receives the signed XY proxy (and with 4 columns the sum
    of per-pixel XY gradient norms in column 3)."""
    cm, vm, uvg, cg, cq, vg, ks, ls, soft = _prepare(
        means3d, color_grads, color_quads, view_grads, specular_ks, specular_log_s, softnesses,
        color_model, view_model, use_view_grads)
    if return_overdraw_hits and not return_overdraw:
        raise ValueError("return_overdraw_hits requires return_overdraw=True")
    if return_distortion and not return_surface:
        raise ValueError("return_distortion requires return_surface=True")
    if return_median_depth and not return_surface:
        raise ValueError("Median depth requires surface outputs")
    means2d_in = means2d.contiguous() if means2d is not None else _empty_like(means3d)
    opts = dict(image_width=int(image_width), image_height=int(image_height),
                tan_fovx=float(tan_fovx), tan_fovy=float(tan_fovy), softness=float(softness),
                scale_modifier=float(scale_modifier), color_model=cm, view_model=vm,
                use_view_grads=uvg, prefilter_edge_on=bool(prefilter_edge_on),
                conservative_bounds=bool(conservative_bounds), debug=bool(debug),
                return_contrib=bool(return_contrib), return_overdraw=bool(return_overdraw),
                return_overdraw_hits=bool(return_overdraw_hits),
                return_surface=bool(return_surface), overdraw_base_count=int(overdraw_base_count),
                return_median_depth=bool(return_median_depth))
    out = _RasterizeHexels3D.apply(
        means3d.contiguous(), means2d_in, scales.contiguous(), rotations.contiguous(),
        colors.contiguous(), cg, cq, vg, ks, ls, opacities.contiguous(), soft,
        viewmatrix.contiguous(), projmatrix.contiguous(), campos.contiguous(),
        background.contiguous(), opts)
    out_color, radii, contrib, overdraw, overdraw_hits, depth, alpha, maps = out
    outputs = [out_color, radii]
    if return_contrib:
        outputs.append(contrib)
    if return_overdraw:
        outputs.append(overdraw)
    if return_overdraw_hits:
        outputs.append(overdraw_hits)
    if return_surface:
        outputs.extend([depth, alpha, maps[:3]])
        if return_distortion:
            outputs.append(maps[3])
        if return_median_depth:
            outputs.append(maps[4])
    return tuple(outputs)


def _with(return_contrib, return_overdraw):
    def fn(means3d, scales, rotations, colors, color_grads, view_grads, opacities, viewmatrix,
           projmatrix, campos, background, image_width, image_height, tan_fovx, tan_fovy,
           softness, softnesses=None, *, color_quads=None, scale_modifier=1.0,
           color_model="linear", use_view_grads=True, debug=False):
        return rasterize_hexels3d(
            means3d, scales, rotations, colors, color_grads, view_grads, opacities, viewmatrix,
            projmatrix, campos, background, image_width, image_height, tan_fovx, tan_fovy,
            softness, softnesses, color_quads=color_quads, scale_modifier=scale_modifier,
            color_model=color_model, use_view_grads=use_view_grads,
            return_contrib=return_contrib, return_overdraw=return_overdraw, debug=debug)

    return fn


rasterize_hexels3d_with_contrib = _with(True, False)
rasterize_hexels3d_with_contrib.__name__ = "rasterize_hexels3d_with_contrib"
rasterize_hexels3d_with_overdraw = _with(False, True)
rasterize_hexels3d_with_overdraw.__name__ = "rasterize_hexels3d_with_overdraw"
rasterize_hexels3d_with_contrib_overdraw = _with(True, True)
rasterize_hexels3d_with_contrib_overdraw.__name__ = "rasterize_hexels3d_with_contrib_overdraw"


class Hexels3DRasterizer(torch.nn.Module):
    """Module wrapper holding the camera intrinsics and appearance options
    (reference gsplat/rasterize_hexels3d.py:2494-2638)."""

    def __init__(self, image_width: int, image_height: int, tan_fovx: float, tan_fovy: float,
                 softness: float, scale_modifier: float = 1.0, *,
                 color_model: ColorModel = "linear", view_model: ViewModel = "linear",
                 use_view_grads: bool = True, debug: bool = False) -> None:
        super().__init__()
        self.image_width = int(image_width)
        self.image_height = int(image_height)
        self.tan_fovx = float(tan_fovx)
        self.tan_fovy = float(tan_fovy)
        self.softness = float(softness)
        self.scale_modifier = float(scale_modifier)
        self.color_model = str(color_model)
        self.view_model = str(view_model)
        self.use_view_grads = bool(use_view_grads)
        self.debug = bool(debug)

    def _common(self):
        return dict(image_width=self.image_width, image_height=self.image_height,
                    tan_fovx=self.tan_fovx, tan_fovy=self.tan_fovy, softness=self.softness)

    def render_owner(self, means3d, scales, rotations, colors, color_grads, view_grads, opacities,
                     viewmatrix, projmatrix, campos, background, *, color_quads=None,
                     specular_ks=None, specular_log_s=None, softnesses=None,
                     prefilter_edge_on=False, conservative_bounds=False):
        return rasterize_hexels3d_owner_forward(
            means3d, scales, rotations, colors, color_grads, view_grads, opacities, viewmatrix,
            projmatrix, campos, background, softnesses=softnesses, color_quads=color_quads,
            specular_ks=specular_ks, specular_log_s=specular_log_s,
            scale_modifier=self.scale_modifier, color_model=self.color_model,
            view_model=self.view_model, use_view_grads=self.use_view_grads,
            prefilter_edge_on=prefilter_edge_on, conservative_bounds=conservative_bounds,
            debug=self.debug, **self._common())

    def forward(self, means3d, scales, rotations, colors, color_grads, view_grads, opacities,
                viewmatrix, projmatrix, campos, background, *, means2d=None, color_quads=None,
                specular_ks=None, specular_log_s=None, softnesses=None, return_contrib=False,
                return_overdraw=False, return_overdraw_hits=False, return_surface=False,
                return_distortion=False, return_median_depth=False, overdraw_base_count=-1,
                prefilter_edge_on=False, conservative_bounds=False):
        return rasterize_hexels3d(
            means3d, scales, rotations, colors, color_grads, view_grads, opacities, viewmatrix,
            projmatrix, campos, background, softnesses=softnesses, means2d=means2d,
            color_quads=color_quads, specular_ks=specular_ks, specular_log_s=specular_log_s,
            scale_modifier=self.scale_modifier, color_model=self.color_model,
            view_model=self.view_model, use_view_grads=self.use_view_grads,
            return_contrib=return_contrib, return_overdraw=return_overdraw,
            return_overdraw_hits=return_overdraw_hits, return_surface=return_surface,
            return_distortion=return_distortion, return_median_depth=return_median_depth,
            overdraw_base_count=overdraw_base_count, prefilter_edge_on=prefilter_edge_on,
            conservative_bounds=conservative_bounds, debug=self.debug, **self._common())


__all__ = [
    "Hexels3DRasterizer",
    "rasterize_hexels3d",
    "rasterize_hexels3d_owner_forward",
    "rasterize_hexels3d_forward",
    "rasterize_hexels3d_forward_with_contrib",
    "rasterize_hexels3d_forward_with_overdraw",
    "rasterize_hexels3d_forward_with_overdraw_hits",
    "rasterize_hexels3d_forward_with_contrib_overdraw",
    "rasterize_hexels3d_forward_with_contrib_overdraw_hits",
    "rasterize_hexels3d_exact_sort_forward",
    "rasterize_hexels3d_pixel_risk_forward",
    "rasterize_hexels3d_with_contrib",
    "rasterize_hexels3d_with_overdraw",
    "rasterize_hexels3d_with_contrib_overdraw",
]
