"""One fit step over several views of one 3D hexel-surfel scene, the views
pipelined over CUDA streams.

Within a step the surfel parameters are fixed, so the views are independent
until their gradients meet: view v + 1's preprocess, depth order and binning
(short, latency-bound kernels) and its compositing can run while view v's
compositing finishes, filling the idle tails of each launch.  Views are dealt
to `streams` CUDA streams in turn.  The compositing backward adds colour,
colour-gradient, view-gradient and opacity gradients with atomics, so all
streams share those accumulators; the geometry backward adds the means,
scales and rotations gradients without atomics, so every stream but the first
gets private accumulators, added into the caller's after the step.  The
colour loss of each view (mean squared error to its target) is added into one
loss slot by the fused loss kernel.

The per-view work is the cached forward and backward of
gsplat.cuda_hexels3d._C (the kernels behind gsplat.rasterize_hexels3d), RGB
outputs only.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

PARAM_NAMES = ("means3d", "scales", "rotations", "colors", "color_grads", "view_grads",
               "opacities")


class ViewPipeline:
    """Streams and private geometry accumulators reused across steps."""

    def __init__(self, params: Sequence[torch.Tensor], streams: int = 2):
        if streams < 1:
            raise ValueError("streams must be >= 1")
        self.streams = [torch.cuda.Stream(device=params[0].device) for _ in range(streams)]
        # means3d, scales and rotations accumulators of streams 1.. (stream 0
        # uses the caller's)
        self.geo = [[torch.zeros_like(p) for p in params[:3]] for _ in range(streams - 1)]


def view_groups(n_views: int, group: int) -> list:
    """Group sizes of a rank's views for fit_step_views: groups of
    at most `group` views and at most half of the views each, so that both
    streams have a group to overlap (8 views of 1080p on one GPU: 16.19 ms as
    2 groups of 4, 16.63 ms as 1 group of 8; a separate first group of 2
    views, whose binning nothing overlaps, measured no faster: 15.39 against
    15.30 ms for 8 views, 115.4 against 115.1 ms for 64)."""
    if n_views <= 0:
        return []
    cap = max(1, min(group, (n_views + 1) // 2))
    k = -(-n_views // cap)
    return [n_views // k + (1 if i < n_views % k else 0) for i in range(k)]


def fit_step_views(params: Sequence[torch.Tensor], cams: Sequence, targets: Sequence[torch.Tensor],
                   background: torch.Tensor, softness: float, grads: Sequence[torch.Tensor],
                   loss: torch.Tensor, pipeline: Optional[ViewPipeline] = None, *,
                   color_model: int = 1, view_model: int = 1,
                   use_view_grads: bool = True, group=1) -> None:
    """Forward, loss and backward of every view in `cams` (objects with
    viewmatrix, projmatrix, campos, width, height, tan_fovx, tan_fovy), the
    gradients of `params` (means3d, scales, rotations, colors, color_grads,
    view_grads, opacities) ADDED into `grads` (same order and shapes) and the
    summed per-view colour losses ADDED into `loss` (one element).  With a
    `pipeline` of several streams the views run overlapped; without one they
    run in order on the current stream.  With `group` > 1 the views are taken
    `group` at a time (or, with a sequence, in groups of those sizes, which
    sum to the number of views) and each group is binned together
    (_C._forward_views_core: one depth order, one binning and one read-back
    of the intersection count per group instead of per view); the groups are
    dealt to the streams.  Each view's intermediate tensors are made and used
    on one stream only, so the caching allocator reuses them in that
    stream's order; the accumulators are the caller's and the current stream
    waits for every view before this returns."""
    from gsplat.cuda_hexels3d import _C
    from gsplat.loss import l2_loss_grad

    if len(params) != 7 or len(grads) != 7:
        raise ValueError("params and grads take the 7 tensors " + ", ".join(PARAM_NAMES))
    if len(cams) != len(targets):
        raise ValueError("one target per camera")
    if isinstance(group, int):
        if group < 1:
            raise ValueError("group must be >= 1")
        sizes = [min(group, len(cams) - g0) for g0 in range(0, len(cams), group)]
    else:
        sizes = [int(n) for n in group]
        if any(n < 1 for n in sizes) or sum(sizes) != len(cams):
            raise ValueError("group sizes must be >= 1 and sum to the number of views")
    m3, sc, rot, col, cg, vg, op = params
    e = torch.empty(0, device=m3.device)
    main = torch.cuda.current_stream(m3.device)
    streams = pipeline.streams if pipeline is not None else [main]
    if pipeline is not None:
        for acc in pipeline.geo:
            for t in acc:
                t.zero_()
        for s in streams:
            s.wait_stream(main)
    grouped = len(sizes) < len(cams)  # groups of one view take the per-view path
    if grouped:
        g0 = 0
        for gi, n in enumerate(sizes):
            k = gi % len(streams)
            acc = dict(zip(PARAM_NAMES, grads))
            if k > 0:
                acc.update(zip(PARAM_NAMES[:3], pipeline.geo[k - 1]))
            with torch.cuda.stream(streams[k]):
                outs = _C._forward_views_core(m3, sc, rot, col, cg, vg, op, cams[g0:g0 + n],
                                              background, softness, color_model, view_model,
                                              use_view_grads)
                for o, cam, tgt in zip(outs, cams[g0:g0 + n], targets[g0:g0 + n]):
                    _, g_color = l2_loss_grad(o["out_color"], tgt, loss=loss)
                    _C._backward_core(m3, e, sc, rot, col, cg, e, vg, e, e, op, e,
                                      cam.viewmatrix, cam.projmatrix, cam.campos, background,
                                      g_color, e, e, e, e, cam.width, cam.height, cam.tan_fovx,
                                      cam.tan_fovy, softness, 1.0, color_model, view_model,
                                      use_view_grads, -1, False, False, False, o["saved"],
                                      accumulate_into=acc, blend_mask=o["blend_mask"],
                                      records=o["records"])
                    del g_color
                del outs
            g0 += n
    for i, (cam, tgt) in enumerate(zip(cams, targets) if not grouped else ()):
        k = i % len(streams)
        acc = dict(zip(PARAM_NAMES, grads))
        if k > 0:
            acc.update(zip(PARAM_NAMES[:3], pipeline.geo[k - 1]))
        with torch.cuda.stream(streams[k]):
            o = _C._forward_core(m3, sc, rot, col, cg, e, vg, e, e, op, e, cam.viewmatrix,
                                 cam.projmatrix, cam.campos, background, cam.width, cam.height,
                                 cam.tan_fovx, cam.tan_fovy, softness, 1.0, color_model,
                                 view_model, use_view_grads, False, False, False, save=True)
            _, g_color = l2_loss_grad(o["out_color"], tgt, loss=loss)
            _C._backward_core(m3, e, sc, rot, col, cg, e, vg, e, e, op, e, cam.viewmatrix,
                              cam.projmatrix, cam.campos, background, g_color, e, e, e, e,
                              cam.width, cam.height, cam.tan_fovx, cam.tan_fovy, softness, 1.0,
                              color_model, view_model, use_view_grads, -1, False, False, False,
                              o["saved"], accumulate_into=acc, blend_mask=o["blend_mask"],
                              records=o["records"])
            del o, g_color
    if pipeline is not None:
        for s in streams:
            main.wait_stream(s)
        for acc in pipeline.geo:
            for dst, src in zip(grads[:3], acc):
                dst.add_(src)
