"""Parity against the reference's own CUDA kernels (oracle/_ref, compiled from
its sources) at the sizes the benchmark configurations are quoted on:

  * 3D single view, 1,000,000 surfels at 1920x1080 with depth/normal outputs
    (forward_all + the uncached backward);
  * 3D multi-view, the same scene from orbit views 0 and 17 on the cached RGB
    path (forward_cached's eleven saved buffers + backward_cached);
  * Image-GS large, 2048x2048 with 100,000 Gaussians, top-10 (projection,
    binning, compositing, backward, projection VJP);
  * 2D image hexels, 1024x1024 with 50,000 hexagons, top-10.

Tolerances: integer outputs (radii, tile counts, intersection counts, keys,
sorted lists, tile ranges, last indices, top-K ids) and the projection's
float outputs bit-exact; images and per-pixel float state 1e-5 absolute
(scaled by the channel's largest magnitude for depth).  Gradients: the stated
criterion (1e-4 relative, 1e-6 absolute near zero) is not met by the
reference against a second run of itself at these sizes (float32 atomics in
another order), so conftest.assert_grad_at_size gates ours by the
reference's own count of entries outside it and settles the worst entries
against the float64 oracle.  The upstream gradients are seeded U[-1,1) per
pixel so that every gradient is of order one and the absolute floor is
tight.  Each test prints its figures (run with -rP to see them).
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import assert_grad_at_size, grad_compare_at_size, ref_module

pytestmark = pytest.mark.gpu
IMG_ATOL = 1e-5

GRAD_NAMES = ("means3d", "means2d", "scales", "rotations", "colors", "color_grads",
              "color_quads", "view_grads", "specular_ks", "specular_log_s", "opacities",
              "softnesses")
SAVED_NAMES = ("radii", "transMats", "opacities", "softnesses", "view_dirs", "normals",
               "points_xy_center", "ranges", "point_list", "final_T", "last_index")


@pytest.fixture(scope="module")
def ref3d():
    r = ref_module("_ref_hexels3d_C")
    if r is None:
        pytest.skip("reference kernels not built")
    return r


@pytest.fixture(scope="module")
def ref2d():
    r = ref_module("_ref_gsplat_csrc")
    if r is None:
        pytest.skip("reference kernels not built")
    return r


def _upstream(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(shape, generator=g) * 2 - 1).cuda()


def _compare(names, mine, theirs, again):
    return [grad_compare_at_size(a, b, c, n) for n, a, b, c in zip(names, mine, theirs, again)]


def _settle(title, stats, exact_fn=None, row_width=None):
    """Print and assert each tensor's figures.  With `exact_fn`, the worst
    entries outside the stated criterion are settled against the float64
    oracle (`exact_fn(rows)` -> {name: ((len(rows), k) float64 tensor,
    (len(rows), k) float32 tensor)})."""
    row_width = row_width or {}
    rows = sorted({i // row_width[st["name"]] for st in stats
                   if st.get("worst") and st["name"] in row_width for i in st["worst"]})
    exact = exact_fn(rows) if rows and exact_fn is not None else {}
    pos = {r: k for k, r in enumerate(rows)}
    print(f"\n[{title}]")
    failures = []
    for st in stats:
        ex = None
        if st.get("worst") and st["name"] in exact:
            wdt = row_width[st["name"]]
            e64, e32 = exact[st["name"]]
            ex = {i: (float(e64[pos[i // wdt]].reshape(-1)[i % wdt]),
                      float(e32[pos[i // wdt]].reshape(-1)[i % wdt])) for i in st["worst"]}
        try:
            assert_grad_at_size(st, ex)
        except AssertionError as err:
            failures.append(str(err))
        st.pop("_tensors", None)
        print(json.dumps(st))
    assert not failures, "; ".join(failures)


# ---------------------------------------------------------------------------
# 3D hexel surfels
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def scene3d():
    import workloads

    w = workloads.hexels3d_multiview(64)
    dev = "cuda"
    return dict(
        w=w,
        params=tuple(t.to(dev) for t in (w.means3d, w.scales, w.rotations, w.colors,
                                         w.color_grads, w.view_grads, w.opacities)),
        bg=w.background.to(dev))


def _tens(scene, cam):
    m3, sc, rot, col, cg, vg, op = scene["params"]
    e = torch.empty(0, device="cuda")
    t = (m3, sc, rot, col, cg, e, vg, e, e, op, e, cam.viewmatrix, cam.projmatrix, cam.campos,
         scene["bg"])
    s = (cam.width, cam.height, cam.tan_fovx, cam.tan_fovy, scene["w"].softness, 1.0, 1, 1, True)
    return t, s


ROW3D = {"means3d": 3, "scales": 2, "rotations": 4, "colors": 3, "color_grads": 6,
         "view_grads": 9, "opacities": 1}


def _exact_3d(scene, cam, saved, radii, upstream, surfels, surface=False, normals=None):
    """Oracle gradients of the given surfels in float64 and in float32.  A
    surfel's gradient sums over the pixels of the tiles whose lists hold it,
    so only those tiles are composited (all their surfels, from the GPU's
    preprocess state), then the geometry VJP maps the transform, view
    direction and normal gradients to means3d, scales and rotations."""
    from oracle import hexels3d as o

    w = scene["w"]
    m3, sc, rot, col, cg, vg, op = (t.cpu() for t in scene["params"])
    W, H = cam.width, cam.height
    grid = ((W + 15) // 16, (H + 15) // 16)
    ranges = saved[7].cpu().numpy().astype(np.int64)
    plist = saved[8].cpu().numpy()
    tile_of = np.repeat(np.arange(grid[0] * grid[1]), ranges[:, 1] - ranges[:, 0])
    tiles = np.unique(tile_of[np.isin(plist, np.asarray(surfels))])
    pre = dict(transMats=saved[1].cpu(), opacities=saved[2].cpu(), softnesses=saved[3].cpu(),
               softness_stride=1, view_dirs=saved[4].cpu(),
               normals=normals.cpu() if normals is not None else o.normals_of(rot),
               points_xy_center=torch.zeros((w.num_points, 2)), W=W, H=H, grid=grid)
    idx = torch.as_tensor(surfels, dtype=torch.long)
    out = {}
    for dt in (torch.float64, torch.float32):
        o.set_precision(dt)
        try:
            r = o.render(pre, ranges, plist, col, scene["bg"].cpu(), cg, None, vg, None, None, 1,
                         1, True, surface=surface, tiles=tiles,
                         upstream={k: v.cpu() for k, v in upstream.items()})
            G = r["grads"]
            gm, gs, gq = o.geometry_backward(m3, sc, rot, cam.projmatrix.cpu(), cam.campos.cpu(),
                                             W, H, radii.cpu().numpy(), G["transMats"],
                                             G["view_dirs"], G["normals"] if surface else None)
        finally:
            o.set_precision(torch.float32)
        full = {"means3d": gm, "scales": gs, "rotations": gq, "colors": G["colors"],
                "color_grads": G["color_grads"], "view_grads": G["view_grads"],
                "opacities": G["opacities"]}
        for k, v in full.items():
            out.setdefault(k, []).append(v.reshape(w.num_points, -1)[idx].double())
    return {k: tuple(v) for k, v in out.items()}


@pytest.mark.parametrize("view", [0, 17])
def test_multiview_cached_path_matches_reference(ref3d, scene3d, view):
    """One orbit view of the 64-view 1M-surfel scene on the cached RGB
    training path: the eleven saved buffers (radii, transforms, tile ranges,
    the sorted surfel list, last indices ...) bit-exact, the image within
    1e-5, and the cached backward's gradients in tolerance."""
    from gsplat.cuda_hexels3d import _C

    cam = scene3d["w"].cameras[view].to("cuda")
    t, s = _tens(scene3d, cam)
    mine = _C.rasterize_hexels3d_forward_cached(*t, *s, False, False, False)
    theirs = ref3d.rasterize_hexels3d_forward_cached(*t, *s, False, False, False)
    n_rendered = theirs[2][8].numel()
    assert n_rendered > 1_000_000
    for n, a, b in zip(SAVED_NAMES, mine[2], theirs[2]):
        assert a.shape == b.shape and a.dtype == b.dtype, n
        if n == "final_T":
            torch.testing.assert_close(a, b, rtol=0, atol=IMG_ATOL, msg=n)
        else:
            assert torch.equal(a, b), f"{n}: {int((a != b).sum())} entries differ"
    torch.testing.assert_close(mine[0], theirs[0], rtol=0, atol=IMG_ATOL)
    assert torch.equal(mine[1], theirs[1])

    H, W = cam.height, cam.width
    gc = _upstream((3, H, W), 100 + view)
    e = torch.empty(0, device="cuda")
    bargs = (t[0], e, *t[1:], gc, e, e, e, e, *s, -1, False, False, False)
    gm = _C.rasterize_hexels3d_backward_cached(*bargs, list(mine[2]))
    gr = ref3d.rasterize_hexels3d_backward_cached(*bargs, list(theirs[2]))
    gr2 = ref3d.rasterize_hexels3d_backward_cached(*bargs, list(theirs[2]))
    stats = _compare(GRAD_NAMES, gm, gr, gr2)
    _settle(f"c5 view {view}: {n_rendered} intersections", stats, lambda surfels: _exact_3d(
        scene3d, cam, mine[2], mine[1], {"color": gc.reshape(3, -1)}, surfels), ROW3D)


def test_single_view_surface_matches_reference(ref3d, scene3d):
    """The single-view configuration (view 0, 1M surfels, 1920x1080) with
    depth and normal outputs: forward_all's outputs, then the uncached
    backward with colour, depth, alpha and normal (+ distortion) gradients."""
    from gsplat.cuda_hexels3d import _C

    cam = scene3d["w"].cameras[0].to("cuda")
    t, s = _tens(scene3d, cam)
    flags = (False, False, False, True, -1, False, False, False)
    mine = _C.rasterize_hexels3d_forward_all(*t, *s, *flags)
    theirs = ref3d.rasterize_hexels3d_forward_all(*t, *s, *flags)
    names = ("out_color", "radii", "contrib", "overdraw", "overdraw_hits", "depth", "alpha",
             "surface")
    for n, a, b in zip(names, mine, theirs):
        assert a.shape == b.shape, n
        if a.dtype.is_floating_point:
            scale = max(1.0, float(b.abs().max())) if b.numel() else 1.0
            torch.testing.assert_close(a, b, rtol=0, atol=IMG_ATOL * scale, msg=n)
        else:
            assert torch.equal(a, b), n

    H, W = cam.height, cam.width
    gc = _upstream((3, H, W), 200)
    gd = _upstream((H, W), 201)
    ga = _upstream((H, W), 202)
    gn = _upstream((4, H, W), 203)
    e = torch.empty(0, device="cuda")
    bargs = (t[0], e, *t[1:], gc, e, gd, ga, gn, *s, -1, False, False, False)
    gm = _C.rasterize_hexels3d_backward(*bargs)
    gr = ref3d.rasterize_hexels3d_backward(*bargs)
    gr2 = ref3d.rasterize_hexels3d_backward(*bargs)
    stats = _compare(GRAD_NAMES, gm, gr, gr2)
    f = _C._forward_core(*t, *s, False, False, False, return_surface=True, save=True,
                         save_surface=True)
    up = {"color": gc.reshape(3, -1), "depth": gd.reshape(-1), "alpha": ga.reshape(-1),
          "normal": gn[:3].reshape(3, -1), "distortion": gn[3].reshape(-1)}
    _settle("c4 view 0, surface outputs", stats, lambda surfels: _exact_3d(
        scene3d, cam, f["saved"], f["radii"], up, surfels, surface=True,
        normals=f["normals"]), ROW3D)


# ---------------------------------------------------------------------------
# Image-GS, 2048x2048, 100,000 Gaussians, top-10
# ---------------------------------------------------------------------------
def test_imagegs_large_matches_reference(ref2d):
    import gsplat
    import workloads
    from gsplat import csrc

    w = workloads.imagegs_large()
    m, sc, rot, col = (t.cuda() for t in (w.means2d, w.scales2d, w.rotation, w.colors))
    H, W, tb, n = w.height, w.width, w.tile_bounds, w.num_points
    T = tb[0] * tb[1]

    xys, radii, conics, nth = csrc.project_gaussians_2d_scale_rot_forward(n, m, sc, rot, H, W, tb)
    r = ref2d.project_gaussians_2d_scale_rot_forward(n, m, sc, rot, H, W, tb)
    for name, a, b in zip(("xys", "radii", "conics", "num_tiles_hit"), (xys, radii, conics, nth),
                          r):
        assert torch.equal(a, b), name

    # binning: ours against the reference's own sequence (utils.py:96-162)
    n_isect, cum = gsplat.compute_cumulative_intersects(nth)
    isect, gids, isect_s, gids_s, bins = gsplat.bin_and_sort_gaussians(n, n_isect, xys, radii,
                                                                       cum, tb)
    r_cum = torch.cumsum(r[3], dim=0, dtype=torch.int32)
    assert n_isect == int(r_cum[-1]) and torch.equal(cum, r_cum)
    r_isect, r_gids = ref2d.map_gaussian_to_intersects(n, n_isect, xys, radii, r_cum, tb)
    assert torch.equal(isect, r_isect) and torch.equal(gids, r_gids)
    r_sorted, order = torch.sort(r_isect)
    r_gsorted = torch.gather(r_gids, 0, order)
    r_bins = ref2d.get_tile_bin_edges(n_isect, T, r_sorted)
    assert torch.equal(isect_s, r_sorted)
    assert torch.equal(bins, r_bins)
    # id order within a tile: stable here; torch.sort's is unspecified by API
    b_np = bins.cpu().numpy()
    same_ids = (gids_s == r_gsorted).cpu().numpy()
    tiles_same = np.array([same_ids[a:b].all() for a, b in b_np])
    frac_tiles_same = float(tiles_same.mean())

    img, topk = csrc.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (W, H, 1), gids_s, bins, xys,
                                                    conics, col)
    r_img, r_topk = ref2d.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (W, H, 1), r_gsorted,
                                                         r_bins, xys, conics, col)
    # pixels of tiles whose id order agrees must have identical top-K lists
    px_tile = (torch.arange(H).view(H, 1) // 16 * tb[0] + torch.arange(W).view(1, W) // 16)
    px_same = torch.from_numpy(tiles_same)[px_tile].cuda()
    assert torch.equal(topk[px_same], r_topk[px_same])
    frac_topk_equal = float((topk == r_topk).all(-1).float().mean())
    torch.testing.assert_close(img[px_same], r_img[px_same], rtol=0, atol=IMG_ATOL)

    v_out = _upstream(img.shape, 300)
    gm = csrc.nd_rasterize_backward_topk_norm(H, W, 16, 16, gids_s, bins, xys, conics, col, v_out,
                                              topk)
    gr = ref2d.nd_rasterize_backward_topk_norm(H, W, 16, 16, r_gsorted, r_bins, xys, conics, col,
                                               v_out, r_topk)
    gr2 = ref2d.nd_rasterize_backward_topk_norm(H, W, 16, 16, r_gsorted, r_bins, xys, conics,
                                                col, v_out, r_topk)
    stats = _compare(("v_xy", "v_conic", "v_colors"), gm, gr, gr2)
    pm = csrc.project_gaussians_2d_scale_rot_backward(n, m, sc, rot, H, W, radii, conics, gm[0],
                                                      gm[1])
    pr = ref2d.project_gaussians_2d_scale_rot_backward(n, m, sc, rot, H, W, radii, conics, gr[0],
                                                       gr[1])
    pr2 = ref2d.project_gaussians_2d_scale_rot_backward(n, m, sc, rot, H, W, radii, conics,
                                                        gr2[0], gr2[1])
    stats += _compare(("v_cov2d", "v_mean2d", "v_scale", "v_rot"), pm, pr, pr2)
    print(json.dumps({"intersections": n_isect, "tiles_with_torch_sort_order": frac_tiles_same,
                      "pixels_topk_equal": frac_topk_equal}))
    _settle("c2 Image-GS 2048x2048 / 100k", stats)


# ---------------------------------------------------------------------------
# 2D image hexels, 1024x1024, 50,000 hexagons, top-10
# ---------------------------------------------------------------------------
def test_hexels2d_matches_reference(ref2d):
    import gsplat
    import workloads
    from gsplat import csrc
    from gsplat.utils import count_tiles_in_rows

    w = workloads.hexels2d()
    xys, scales, rot, col, radii = (t.cuda() for t in (w.xys, w.scales, w.rotation, w.colors,
                                                      w.radii))
    H, W, tb, n = w.height, w.width, w.tile_bounds, w.num_points
    T = tb[0] * tb[1]
    e = torch.empty(0, device="cuda")
    nth = count_tiles_in_rows(xys, radii, tb, (0, tb[1]))
    n_isect, cum = gsplat.compute_cumulative_intersects(nth)
    _, _, isect_s, gids_s, bins = gsplat.bin_and_sort_gaussians(n, n_isect, xys, radii, cum, tb)
    r_cum = torch.cumsum(nth, dim=0, dtype=torch.int32)
    r_isect, r_gids = ref2d.map_gaussian_to_intersects(n, n_isect, xys, radii, r_cum, tb)
    r_sorted, order = torch.sort(r_isect)
    r_gsorted = torch.gather(r_gids, 0, order)
    r_bins = ref2d.get_tile_bin_edges(n_isect, T, r_sorted)
    assert torch.equal(isect_s, r_sorted) and torch.equal(bins, r_bins)
    b_np = bins.cpu().numpy()
    same_ids = (gids_s == r_gsorted).cpu().numpy()
    tiles_same = np.array([same_ids[a:b].all() for a, b in b_np])

    fwd = (tb, (16, 16, 1), (W, H, 1))
    img, topk, ws, ent = csrc.nd_rasterize_forward_topk_norm_hexels(
        *fwd, gids_s, bins, xys, scales, rot, col, w.aa_kernel_size, w.softness, e, e)
    r_img, r_topk, r_ws, r_ent = ref2d.nd_rasterize_forward_topk_norm_hexels(
        *fwd, r_gsorted, r_bins, xys, scales, rot, col, w.aa_kernel_size, w.softness, e, e)
    px_tile = (torch.arange(H).view(H, 1) // 16 * tb[0] + torch.arange(W).view(1, W) // 16)
    px_same = torch.from_numpy(tiles_same)[px_tile].cuda()
    assert torch.equal(topk[px_same], r_topk[px_same])
    for name, a, b in (("image", img, r_img), ("weights_sum", ws, r_ws), ("entropy", ent, r_ent)):
        torch.testing.assert_close(a[px_same], b[px_same], rtol=0, atol=IMG_ATOL, msg=name)

    v_out = _upstream(img.shape, 400)
    v_ws = _upstream((H, W), 401) * 0.1
    v_en = _upstream((H, W), 402) * 0.1
    bwd = (H, W, 16, 16)
    gm = csrc.nd_rasterize_backward_topk_norm_hexels(
        *bwd, gids_s, bins, xys, scales, rot, col, v_out, v_ws, v_en, topk, w.aa_kernel_size,
        w.softness, e, e)
    gr = ref2d.nd_rasterize_backward_topk_norm_hexels(
        *bwd, r_gsorted, r_bins, xys, scales, rot, col, v_out, v_ws, v_en, r_topk,
        w.aa_kernel_size, w.softness, e, e)
    gr2 = ref2d.nd_rasterize_backward_topk_norm_hexels(
        *bwd, r_gsorted, r_bins, xys, scales, rot, col, v_out, v_ws, v_en, r_topk,
        w.aa_kernel_size, w.softness, e, e)
    # (v_emission and v_sharpness are empty: neither term is an input here)
    stats = _compare(("v_xy", "v_scale", "v_rot", "v_colors"), gm[:4], gr[:4], gr2[:4])
    print(json.dumps({"intersections": n_isect,
                      "tiles_with_torch_sort_order": float(tiles_same.mean()),
                      "pixels_topk_equal": float((topk == r_topk).all(-1).float().mean())}))
    _settle("c3 2D hexels 1024x1024 / 50k", stats)
