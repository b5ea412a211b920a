"""GPU parity of the 3D hexel surfel rasteriser against the reference's own
CUDA kernels (oracle/_ref/_ref_hexels3d_C, compiled from its sources) and the
CPU oracle.

Tolerances: radii, transforms, tile ranges and sorted surfel lists
bit-exact; images and per-pixel outputs 1e-5 absolute; gradients per
conftest.assert_grad_parity (1e-4 relative with a 1e-5 x max|grad| floor).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close_oracle, assert_grad_parity, ref_module

pytestmark = pytest.mark.gpu
IMG_ATOL = 1e-5


@pytest.fixture(scope="module")
def ref():
    return ref_module("_ref_hexels3d_C")


def _scene(seed=1, P=1500, W=88, H=72, scale=0.06, view=0, **kw):
    import workloads

    w = workloads.hexels3d_tiny(seed, P, W, H, 2, scale).to("cuda")
    cam = w.cameras[view]
    g = torch.Generator().manual_seed(seed + 100)
    extra = dict(
        color_quads=(0.05 * torch.randn((P, 3, 3), generator=g)).cuda(),
        specular_ks=(0.2 * torch.rand((P, 3), generator=g)).cuda(),
        specular_log_s=(3 * torch.rand((P,), generator=g) - 0.5).cuda(),
        soft1=(8 + 4 * torch.rand((P,), generator=g)).cuda(),
        soft3=(8 + 4 * torch.rand((P, 3), generator=g)).cuda(),
    )
    return w, cam, extra


def _args(w, cam, extra, color_model=1, view_model=1, softness_kind=None):
    e = torch.empty(0, device="cuda")
    cg = w.color_grads if color_model >= 1 else e
    cq = extra["color_quads"] if color_model >= 2 else e
    uvg = view_model == 1
    vg = w.view_grads if uvg else e
    ks = extra["specular_ks"] if view_model == 2 else e
    ls = extra["specular_log_s"] if view_model == 2 else e
    soft = {None: e, 1: extra["soft1"], 3: extra["soft3"]}[softness_kind]
    tensors = (w.means3d, w.scales, w.rotations, w.colors, cg, cq, vg, ks, ls, w.opacities, soft,
               cam.viewmatrix, cam.projmatrix, cam.campos, w.background)
    scalars = (cam.width, cam.height, cam.tan_fovx, cam.tan_fovy, w.softness, 1.0, color_model,
               view_model, uvg)
    return tensors, scalars


def _grad_outputs(H, W, seed=7, surf_channels=0):
    g = torch.Generator().manual_seed(seed)
    gc = (torch.rand((3, H, W), generator=g) * 2 - 1).cuda()
    if not surf_channels:
        return gc, None
    gd = (torch.rand((H, W), generator=g) * 2 - 1).cuda() * 0.1
    ga = (torch.rand((H, W), generator=g) * 2 - 1).cuda()
    gn = (torch.rand((surf_channels, H, W), generator=g) * 2 - 1).cuda()
    return gc, (gd, ga, gn)


GRAD_NAMES = ("means3d", "means2d", "scales", "rotations", "colors", "color_grads",
              "color_quads", "view_grads", "specular_ks", "specular_log_s", "opacities",
              "softnesses")

CASES = [
    # (color_model, view_model, softness, prefilter, conservative)
    (1, 1, None, False, False),
    (0, 0, None, False, False),
    (1, 1, 3, False, False),
    (1, 1, 1, False, True),
    (2, 1, None, False, False),
    (3, 2, None, False, False),
    (1, 1, None, True, False),
]


@pytest.mark.parametrize("cm,vm,soft,pre,cons", CASES)
def test_cached_forward_backward_matches_reference(ref, cm, vm, soft, pre, cons):
    if ref is None:
        pytest.skip("reference kernels not built")
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene()
    t, s = _args(w, cam, extra, cm, vm, soft)
    mine = _C.rasterize_hexels3d_forward_cached(*t, *s, pre, cons, False)
    theirs = ref.rasterize_hexels3d_forward_cached(*t, *s, pre, cons, False)
    names = ["radii", "transMats", "opacities", "softnesses", "view_dirs", "normals",
             "points_xy_center", "ranges", "point_list", "final_T", "last_index"]
    for n, a, b in zip(names, mine[2], theirs[2]):
        if n in ("final_T",):
            torch.testing.assert_close(a, b, rtol=0, atol=IMG_ATOL, msg=n)
        else:
            assert a.shape == b.shape and torch.equal(a, b), n
    torch.testing.assert_close(mine[0], theirs[0], rtol=0, atol=IMG_ATOL)
    assert torch.equal(mine[1], theirs[1])

    gc, _ = _grad_outputs(cam.height, cam.width)
    e = torch.empty(0, device="cuda")
    means2d = torch.zeros((w.num_points, 4), device="cuda")
    bargs = (t[0], means2d, *t[1:], gc, e, e, e, e, *s, -1, pre, cons, False)
    gm = _C.rasterize_hexels3d_backward_cached(*bargs, list(mine[2]))
    gr = ref.rasterize_hexels3d_backward_cached(*bargs, list(theirs[2]))
    for n, a, b in zip(GRAD_NAMES, gm, gr):
        assert a.shape == b.shape, n
        assert_grad_parity(a, b, None, n)
    # without means2d: the plain-RGB configurations take the backward's
    # 19-component layout
    bargs = (t[0], e, *t[1:], gc, e, e, e, e, *s, -1, pre, cons, False)
    gm = _C.rasterize_hexels3d_backward_cached(*bargs, list(mine[2]))
    gr = ref.rasterize_hexels3d_backward_cached(*bargs, list(theirs[2]))
    for n, a, b in zip(GRAD_NAMES, gm, gr):
        assert a.shape == b.shape, n
        assert_grad_parity(a, b, None, n)


@pytest.mark.parametrize("surface", [False, True])
@pytest.mark.parametrize("cm,vm,soft,pre,cons", CASES)
def test_blend_mask_backward_equals_unmasked(cm, vm, soft, pre, cons, surface):
    """The forward's blend mask only lets the backward skip list entries no
    pixel of a warp's block blends: gradients with and without it agree (to
    the order of the float atomics), and the mask does skip entries."""
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene(seed=8)
    t, s = _args(w, cam, extra, cm, vm, soft)
    H, W = cam.height, cam.width
    f = _C._forward_core(*t, *s, pre, cons, False, return_surface=surface, save=True,
                         save_surface=surface)
    n = f["num_rendered"]
    mask = f["blend_mask"]
    assert mask.dtype == torch.uint8 and mask.numel() >= n
    assert bool((mask[:n] != 0xFF).any())
    gc, surf = _grad_outputs(H, W, seed=3, surf_channels=4 if surface else 0)
    e = torch.empty(0, device="cuda")
    gd, ga, gn = surf if surface else (e, e, e)

    def run(bm):
        return _C._backward_core(t[0], e, *t[1:], gc, e, gd, ga, gn, *s, -1, pre, cons, False,
                                 f["saved"], surf_state=f["surf_state"],
                                 surf_normals=f["normals"] if surface else None, blend_mask=bm)

    for name, a, b in zip(GRAD_NAMES, run(mask), run(None)):
        assert a.shape == b.shape, name
        assert_grad_parity(a, b, None, name)


@pytest.mark.parametrize("median", [False, True])
def test_surface_forward_backward_matches_reference(ref, median):
    if ref is None:
        pytest.skip("reference kernels not built")
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene(seed=2)
    t, s = _args(w, cam, extra)
    fn = "rasterize_hexels3d_forward_median" if median else "rasterize_hexels3d_forward_all"
    flags = (True, True, True, True, -1, False, False, False)
    mine = getattr(_C, fn)(*t, *s, *flags)
    theirs = getattr(ref, fn)(*t, *s, *flags)
    names = ["out_color", "radii", "contrib", "overdraw", "overdraw_hits", "depth", "alpha",
             "surface"]
    for n, a, b in zip(names, mine, theirs):
        assert a.shape == b.shape, n
        if a.dtype.is_floating_point:
            torch.testing.assert_close(a, b, rtol=1e-5, atol=IMG_ATOL * max(1.0, float(
                b.abs().max()) if b.numel() else 1.0), msg=n)
        else:
            assert torch.equal(a, b), n
    gc, (gd, ga, gn) = _grad_outputs(cam.height, cam.width, surf_channels=5 if median else 4)
    means2d = torch.zeros((w.num_points, 3), device="cuda")
    god = (torch.rand((cam.height, cam.width), generator=torch.Generator().manual_seed(3))
           * 0.1).cuda()
    bargs = (t[0], means2d, *t[1:], gc, god, gd, ga, gn, *s, -1, False, False, False)
    gm = _C.rasterize_hexels3d_backward(*bargs)
    gr = ref.rasterize_hexels3d_backward(*bargs)
    for n, a, b in zip(GRAD_NAMES, gm, gr):
        assert a.shape == b.shape, n
        assert_grad_parity(a, b, None, n)


def test_owner_and_overdraw_variants_match_reference(ref):
    if ref is None:
        pytest.skip("reference kernels not built")
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene(seed=3)
    t, s = _args(w, cam, extra)
    a = _C.rasterize_hexels3d_owner_forward(*t, *s, False, False, False)
    b = ref.rasterize_hexels3d_owner_forward(*t, *s, False, False, False)
    for x, y in zip(a, b):
        if x.dtype.is_floating_point:
            torch.testing.assert_close(x, y, rtol=1e-5, atol=IMG_ATOL)
        else:
            assert torch.equal(x, y)
    a = _C.rasterize_hexels3d_forward_with_contrib_overdraw_hits(*t, *s, 700, False, False, False)
    b = ref.rasterize_hexels3d_forward_with_contrib_overdraw_hits(*t, *s, 700, False, False, False)
    for x, y in zip(a, b):
        if x.dtype.is_floating_point:
            torch.testing.assert_close(x, y, rtol=1e-5, atol=IMG_ATOL)
        else:
            assert torch.equal(x, y)


@pytest.mark.parametrize("base", [-1, 700])
def test_plain_surface_forward_matches_reference(ref, base):
    """The surface forward without contribution or overdraw outputs (the
    public API's and the fit steps' call; with every surfel a base surfel it
    runs the plain-RGB instantiation) against the reference's forward_all;
    with a base count below P it takes the generic one."""
    if ref is None:
        pytest.skip("reference kernels not built")
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene(seed=4)
    t, s = _args(w, cam, extra)
    for median in (False, True):
        o = _C._forward_core(*t, *s, False, False, False, return_surface=True,
                             overdraw_base_count=base, return_median_depth=median)
        fn = "rasterize_hexels3d_forward_median" if median else "rasterize_hexels3d_forward_all"
        theirs = getattr(ref, fn)(*t, *s, False, False, False, True, base, False, False, False)
        mine = (o["out_color"], o["radii"], o["surf_depth"], o["surf_alpha"], o["surf_maps"])
        for n, a, b in zip(("out_color", "radii", "depth", "alpha", "surface"), mine,
                           (theirs[0], theirs[1], theirs[5], theirs[6], theirs[7])):
            assert a.shape == b.shape, n
            if a.dtype.is_floating_point:
                torch.testing.assert_close(a, b, rtol=1e-5, atol=IMG_ATOL * max(1.0, float(
                    b.abs().max()) if b.numel() else 1.0), msg=n)
            else:
                assert torch.equal(a, b), n


@pytest.mark.parametrize("surface", [False, True])
def test_plain_forward_equals_generic(surface):
    """Asking for the per-pixel pair counts takes the generic forward; without
    them the training instantiation runs.  Same arithmetic: the images and the
    state saved for the backward are bit-identical, and the counts obey
    0 <= blended <= evaluated, blended <= last index."""
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene(seed=5)
    t, s = _args(w, cam, extra)
    kw = dict(return_surface=surface, save=True, save_surface=surface)
    plain = _C._forward_core(*t, *s, False, False, False, **kw)
    generic = _C._forward_core(*t, *s, False, False, False, count_contrib=True, **kw)
    for n in ("out_color", "surf_depth", "surf_alpha", "surf_maps"):
        assert torch.equal(plain[n], generic[n]), n
    for n, a, b in zip(("final_T", "last_index"), plain["saved"][9:], generic["saved"][9:]):
        assert torch.equal(a, b), n
    counts = generic["contrib_count"]
    blended, evaluated = counts[0], counts[1]
    assert int(blended.min()) >= 0 and bool((blended <= evaluated).all())
    assert bool((blended <= generic["saved"][10]).all())
    assert int(blended.sum()) > 0


def test_public_api_autograd_matches_reference_backward(ref):
    """rasterize_hexels3d(return_surface=True) through autograd, against the
    reference's uncached surface backward on the same upstream gradients."""
    import gsplat

    w, cam, extra = _scene(seed=4)
    leaves = [w.means3d.clone().requires_grad_(), w.scales.clone().requires_grad_(),
              w.rotations.clone().requires_grad_(), w.colors.clone().requires_grad_(),
              w.color_grads.clone().requires_grad_(), w.view_grads.clone().requires_grad_(),
              w.opacities.clone().requires_grad_()]
    m3, sc, rot, col, cg, vg, op = leaves
    out = gsplat.rasterize_hexels3d(m3, sc, rot, col, cg, vg, op, cam.viewmatrix, cam.projmatrix,
                                    cam.campos, w.background, cam.width, cam.height,
                                    cam.tan_fovx, cam.tan_fovy, w.softness, return_surface=True,
                                    return_distortion=True)
    color, radii, depth, alpha, normals, distortion = out
    gc, (gd, ga, gn) = _grad_outputs(cam.height, cam.width, surf_channels=4)
    loss = (color * gc).sum() + (depth * gd).sum() + (alpha * ga).sum() + \
        (normals * gn[:3]).sum() + (distortion * gn[3]).sum()
    loss.backward()
    for x in leaves:
        assert x.grad is not None and torch.isfinite(x.grad).all()
    if ref is None:
        return
    t, s = _args(w, cam, extra)
    e = torch.empty(0, device="cuda")
    bargs = (t[0], e, *t[1:], gc, e, gd, ga, gn, *s, -1, False, False, False)
    gr = ref.rasterize_hexels3d_backward(*bargs)
    pairs = [(m3, gr[0]), (sc, gr[2]), (rot, gr[3]), (col, gr[4]), (cg, gr[5]), (vg, gr[7]),
             (op, gr[10])]
    for (x, r), n in zip(pairs, ("means3d", "scales", "rotations", "colors", "color_grads",
                                 "view_grads", "opacities")):
        assert_grad_parity(x.grad, r, None, n)


def test_empty_scene_matches_reference(ref):
    """All surfels behind the camera: nothing is binned, radii are zero and
    every pixel is the background (the reference still launches its
    compositing over the empty tile ranges)."""
    from gsplat.cuda_hexels3d import _C

    w, cam, extra = _scene(seed=5, P=64)
    t, s = _args(w, cam, extra)
    far = list(t)
    far[0] = t[0] + torch.tensor([0.0, 0.0, 10.0], device="cuda")
    bg = torch.tensor([0.2, 0.3, 0.4], device="cuda")
    far[14] = bg
    img, radii = _C.rasterize_hexels3d_forward(*far, *s, False, False, False)
    assert int(radii.abs().sum()) == 0
    assert torch.equal(img, bg.view(3, 1, 1).expand_as(img))
    if ref is not None:
        r = ref.rasterize_hexels3d_forward(*far, *s, False, False, False)
        assert torch.equal(img, r[0]) and torch.equal(radii, r[1])


def test_full_scene_properties():
    """1M surfels at 1920x1080 (the 3D benchmark scene): sorted keys, ranges
    consistent with the sorted list, deterministic image, finite gradients."""
    import workloads
    from gsplat.cuda_hexels3d import _C

    w = workloads.hexels3d_single().to("cuda")
    cam = w.cameras[0]
    extra = {"color_quads": None, "specular_ks": None, "specular_log_s": None,
             "soft1": None, "soft3": None}
    t, s = _args(w, cam, extra)
    a = _C.rasterize_hexels3d_forward_cached(*t, *s, False, False, False)
    b = _C.rasterize_hexels3d_forward_cached(*t, *s, False, False, False)
    assert torch.equal(a[0], b[0]) and torch.equal(a[2][8], b[2][8])
    ranges = a[2][7].cpu().to(torch.int64)
    lens = ranges[:, 1] - ranges[:, 0]
    assert int(lens.sum()) == a[2][8].numel()
    assert torch.isfinite(a[0]).all()
    _check_ordered_binning_matches_full_keys(w, cam, a[2])


def _check_ordered_binning_matches_full_keys(w, cam, saved):
    """The depth-ordered binning (sort surfels by depth, then only tile bits)
    against the direct stable sort of the reference's (tile << 32 | depth)
    keys: identical point lists and ranges, sorted keys non-decreasing."""
    from gsplat._lib import lib, ptr, stream, workspace

    P, W, H = w.num_points, cam.width, cam.height
    dev = w.means3d.device
    f32 = dict(dtype=torch.float32, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    radii = torch.empty((P,), **i32)
    tile_radii = torch.empty((P, 2), **i32)
    xy = torch.empty((P, 2), **f32)
    depths = torch.empty((P,), **f32)
    tm = torch.empty((P, 9), **f32)
    touched = torch.empty((P,), **i32)
    op_out = torch.empty((P,), **f32)
    soft_out = torch.empty((P,), **f32)
    vd = torch.empty((P, 3), **f32)
    s = stream(dev)
    lib.call("hx_hexels3d_preprocess", P, ptr(w.means3d), ptr(w.scales), 1.0, ptr(w.rotations),
             ptr(w.opacities), None, w.softness, 1, ptr(cam.viewmatrix), ptr(cam.projmatrix),
             ptr(cam.campos), W, H, 0, 0, ptr(radii), ptr(tile_radii), ptr(xy), None,
             ptr(depths), ptr(tm), ptr(touched), ptr(op_out), ptr(soft_out), ptr(vd), None, s)
    offsets = torch.empty((P,), **i32)
    total = torch.zeros((1,), dtype=torch.int64, device=dev)
    ws = workspace(lib.query("hx_scan_workspace_bytes", P), dev)
    lib.call("hx_inclusive_scan_i32", ptr(touched), ptr(offsets), P, ptr(total), ptr(ws),
             ws.numel(), s)
    n = int(total.item())
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    ranges = torch.empty((tiles, 2), **i32)
    plist = torch.empty((n,), **i32)
    keys = torch.empty((n,), dtype=torch.int64, device=dev)
    ws = workspace(lib.query("hx_hexels3d_bin_workspace_bytes", n), dev)
    lib.call("hx_hexels3d_bin", P, n, W, H, ptr(xy), ptr(depths), ptr(offsets), ptr(radii),
             ptr(tile_radii), ptr(keys), ptr(plist), ptr(ranges), ptr(ws), ws.numel(), s)
    assert n == saved[8].numel()
    assert torch.equal(plist, saved[8]) and torch.equal(ranges, saved[7])
    k = keys.cpu()
    assert bool((k[1:] >= k[:-1]).all())


# ---------------------------------------------------------------------------
# against the CPU oracle (oracle/hexels3d.py), on the GPU's own sorted lists
# so that the compositing comparison is isolated from preprocess ulps
# ---------------------------------------------------------------------------
def _oracle_pre(saved, w, cam, stride):
    from oracle import hexels3d as o

    P = w.num_points
    normals = saved[5]
    nr = normals.cpu() if normals.numel() else o.normals_of(w.rotations.cpu().float())
    center = saved[6].cpu() if saved[6].numel() else torch.zeros((P, 2))
    return dict(transMats=saved[1].cpu(), opacities=saved[2].cpu(), softnesses=saved[3].cpu(),
                softness_stride=stride, view_dirs=saved[4].cpu(), normals=nr,
                points_xy_center=center, W=cam.width, H=cam.height,
                grid=((cam.width + 15) // 16, (cam.height + 15) // 16))


def _grad_close_oracle(a, b, name):
    """Gradients against the fp32 CPU oracle: 1e-3 relative with a
    1e-5 x max|grad| floor (fused multiply-adds, intrinsics and summation
    order differ; the bit-level parity is against the reference kernels)."""
    b = b.detach().double().cpu()
    torch.testing.assert_close(a.detach().double().cpu(), b, rtol=1e-3,
                               atol=1e-5 * max(1.0, float(b.abs().max()) if b.numel() else 1.0),
                               msg=name)


def _lists(saved):
    return saved[7].cpu().numpy().astype(np.int64), saved[8].cpu().numpy()


@pytest.mark.parametrize("cm,vm,soft,pre,cons", CASES)
def test_cached_forward_backward_matches_oracle(cm, vm, soft, pre, cons):
    from gsplat.cuda_hexels3d import _C
    from oracle import hexels3d as o

    w, cam, extra = _scene()
    t, s = _args(w, cam, extra, cm, vm, soft)
    img, radii, saved = _C.rasterize_hexels3d_forward_cached(*t, *s, pre, cons, False)
    stride = 3 if soft == 3 else 1
    opre = _oracle_pre(saved, w, cam, stride)
    ranges, plist = _lists(saved)
    gc, _ = _grad_outputs(cam.height, cam.width)
    cpu = lambda x: x.cpu() if x is not None and x.numel() else None  # noqa: E731
    r = o.render(opre, ranges, plist, t[3].cpu(), t[14].cpu(), cpu(t[4]), cpu(t[5]), cpu(t[6]),
                 cpu(t[7]), cpu(t[8]), cm, vm, vm == 1, prefilter=pre,
                 upstream={"color": gc.cpu()})
    HW = cam.width * cam.height
    assert_close_oracle(img.cpu().reshape(3, HW), r["color"], "color")
    assert_close_oracle(saved[9].cpu().reshape(HW), r["final_T"], "final_T")
    same_last = (saved[10].cpu().reshape(HW).long() == r["last_index"]).float().mean()
    assert float(same_last) >= 0.999
    e = torch.empty(0, device="cuda")
    means2d = torch.zeros((w.num_points, 4), device="cuda")
    bargs = (t[0], means2d, *t[1:], gc, e, e, e, e, *s, -1, pre, cons, False)
    g = _C.rasterize_hexels3d_backward_cached(*bargs, list(saved))
    G = r["grads"]
    gm3, gs, gq = o.geometry_backward(
        w.means3d.cpu(), w.scales.cpu(), w.rotations.cpu(), cam.projmatrix.cpu(),
        cam.campos.cpu(), cam.width, cam.height, radii.cpu().numpy(), G["transMats"],
        G["view_dirs"] if "view_dirs" in G else torch.zeros((w.num_points, 3)),
        G["normals"] if vm == 2 else None, G["points_xy_center"] if pre else None)
    pairs = [("means3d", g[0], gm3), ("scales", g[2], gs), ("rotations", g[3], gq),
             ("colors", g[4], G["colors"]), ("opacities", g[10], G["opacities"])]
    if cm >= 1:
        pairs.append(("color_grads", g[5], G["color_grads"]))
    if cm >= 2:
        pairs.append(("color_quads", g[6], G["color_quads"]))
    if vm == 1:
        pairs.append(("view_grads", g[7], G["view_grads"]))
    if vm == 2:
        pairs += [("specular_ks", g[8], G["specular_ks"]),
                  ("specular_log_s", g[9], G["specular_log_s"])]
    if soft:
        pairs.append(("softnesses", g[11], G["softnesses"]))
    proxy = o.means2d_proxy(G["transMats"], opre["transMats"], radii.cpu().numpy(), cam.width,
                            cam.height, G["abs_means2d"])
    pairs.append(("means2d", g[1], proxy))
    for name, a, b in pairs:
        _grad_close_oracle(a, b.reshape(a.shape), name)


@pytest.mark.parametrize("median,pre", [(False, False), (True, False), (True, True)])
def test_surface_outputs_and_grads_match_oracle(median, pre):
    from gsplat.cuda_hexels3d import _C
    from oracle import hexels3d as o

    w, cam, extra = _scene(seed=6)
    t, s = _args(w, cam, extra)
    W, H = cam.width, cam.height
    f = _C._forward_core(*t, *s, pre, False, False, return_surface=True,
                         return_median_depth=median, save=True, save_surface=True)
    saved = f["saved"]
    opre = _oracle_pre(saved, w, cam, 1)
    opre["normals"] = f["normals"].cpu()
    ranges, plist = _lists(saved)
    nch = 5 if median else 4
    gc, (gd, ga, gn) = _grad_outputs(H, W, seed=9, surf_channels=nch)
    up = {"color": gc.cpu(), "depth": gd.cpu(), "alpha": ga.cpu(), "normal": gn[:3].cpu(),
          "distortion": gn[3].cpu()}
    if median:
        up["median"] = gn[4].cpu()
    r = o.render(opre, ranges, plist, t[3].cpu(), t[14].cpu(), t[4].cpu(), None, t[6].cpu(),
                 None, None, 1, 1, True, surface=True, median=median, prefilter=pre,
                 upstream=up)
    HW = W * H
    assert_close_oracle(f["out_color"].cpu().reshape(3, HW), r["color"], "color")
    # depth = w (u Tw.x + v Tw.y + Tw.z) carries the ill-conditioning of (u, v) at
    # depths ~3: relative tolerance
    assert_close_oracle(f["surf_depth"].cpu().reshape(HW), r["depth"], "depth", rtol=2e-4)
    assert_close_oracle(f["surf_alpha"].cpu().reshape(HW), r["alpha"], "alpha")
    maps = f["surf_maps"].cpu().reshape(nch, HW)
    assert_close_oracle(maps[:3], r["normal"], "normal")
    assert_close_oracle(maps[3], r["distortion"], "distortion", rtol=1e-4)
    if median:
        agree = (maps[4] - r["median"]).abs() <= 1e-5 * (1 + r["median"].abs())
        assert float(agree.float().mean()) >= 0.999
    e = torch.empty(0, device="cuda")
    god = torch.zeros((H, W), device="cuda")
    g = _C._backward_core(t[0], e, *t[1:], gc, god, gd, ga, gn, *s, -1, pre, False, False,
                          saved, surf_state=f["surf_state"], surf_normals=f["normals"])
    G = r["grads"]
    gm3, gs, gq = o.geometry_backward(
        w.means3d.cpu(), w.scales.cpu(), w.rotations.cpu(), cam.projmatrix.cpu(),
        cam.campos.cpu(), W, H, saved[0].cpu().numpy(), G["transMats"], G["view_dirs"],
        G["normals"], G["points_xy_center"] if pre else None)
    for name, a, b in [("means3d", g[0], gm3), ("scales", g[2], gs), ("rotations", g[3], gq),
                       ("colors", g[4], G["colors"]), ("color_grads", g[5], G["color_grads"]),
                       ("view_grads", g[7], G["view_grads"]),
                       ("opacities", g[10], G["opacities"])]:
        _grad_close_oracle(a, b.reshape(a.shape), name)


def test_preprocess_matches_oracle():
    """Preprocess on the GPU (fused multiply-adds, fast-math intrinsics)
    against the IEEE CPU restatement: transforms to fp32 rounding, radii and
    tile counts equal for all but ulp-boundary surfels."""
    from gsplat.cuda_hexels3d import _C
    from oracle import hexels3d as o

    w, cam, extra = _scene(seed=7, P=3000)
    t, s = _args(w, cam, extra)
    img, radii, saved = _C.rasterize_hexels3d_forward_cached(*t, *s, False, False, False)
    pre = o.preprocess(w.means3d.cpu(), w.scales.cpu(), w.rotations.cpu(), w.opacities.cpu(),
                       cam.viewmatrix.cpu(), cam.projmatrix.cpu(), cam.campos.cpu(), cam.width,
                       cam.height, w.softness)
    r = radii.cpu().numpy()
    same = r == pre["radii"]
    assert same.mean() >= 0.995 and np.abs(r - pre["radii"]).max() <= 1
    live = torch.from_numpy(same & (r > 0))
    torch.testing.assert_close(saved[1].cpu()[live], pre["transMats"][live], rtol=1e-5, atol=1e-5)
    _, plist = _lists(saved)
    keys, ids, ranges = o.bin_surfels(pre)
    assert abs(len(ids) - len(plist)) <= max(4, len(plist) // 200)


@pytest.mark.parametrize("streams", [2, 3])
def test_pipelined_views_equal_sequential(streams):
    """multiview.fit_step_views with the views spread over several streams
    gives the gradients and loss of the same views run in order (to the
    order of the float atomics)."""
    import multiview
    import workloads

    w = workloads.hexels3d_tiny(11, 2000, 96, 80, 5, 0.06).to("cuda")
    params = [w.means3d, w.scales, w.rotations, w.colors, w.color_grads, w.view_grads,
              w.opacities]
    g = torch.Generator().manual_seed(5)
    cams = w.cameras
    targets = [torch.rand((3, c.height, c.width), generator=g).cuda() for c in cams]

    def step(pipe):
        grads = [torch.zeros_like(p) for p in params]
        loss = torch.zeros(1, device="cuda")
        multiview.fit_step_views(params, cams, targets, w.background, w.softness, grads, loss,
                                 pipe)
        torch.cuda.synchronize()
        return grads, loss

    want_g, want_l = step(None)
    pipe = multiview.ViewPipeline(params, streams=streams)
    for _ in range(2):  # the private accumulators are cleared between steps
        got_g, got_l = step(pipe)
        assert abs(float(got_l) - float(want_l)) <= 1e-5 * abs(float(want_l))
        for name, a, b in zip(multiview.PARAM_NAMES, got_g, want_g):
            assert_grad_parity(a, b, None, name)


@pytest.mark.parametrize("views,size", [(5, "tiny"), (3, "full")])
def test_grouped_views_binning_equals_per_view(views, size):
    """_C._forward_views_core (views binned together: one depth order, one
    binning) gives each view the lists, image and saved state of that view
    run alone through _forward_core: ranges shifted by the entries of the
    views before it, identical point lists, bit-identical images, last
    indices and transforms.  Tiny ragged scene and three orbit views of the
    1M-surfel 1080p scene."""
    import workloads
    from gsplat.cuda_hexels3d import _C

    w = (workloads.hexels3d_tiny(12, 2000, 96, 80, views, 0.06) if size == "tiny"
         else workloads.hexels3d_multiview(64)).to("cuda")
    cams = w.cameras[:views] if size == "tiny" else [w.cameras[v] for v in (0, 21, 42)]
    e = torch.empty(0, device="cuda")
    args = (w.means3d, w.scales, w.rotations, w.colors, w.color_grads, w.view_grads,
            w.opacities)
    outs = _C._forward_views_core(*args, cams, w.background, w.softness)
    base = 0
    for o, cam in zip(outs, cams):
        one = _C._forward_core(w.means3d, w.scales, w.rotations, w.colors, w.color_grads, e,
                               w.view_grads, e, e, w.opacities, e, cam.viewmatrix,
                               cam.projmatrix, cam.campos, w.background, cam.width, cam.height,
                               cam.tan_fovx, cam.tan_fovy, w.softness, 1.0, 1, 1, True, False,
                               False, False, save=True)
        n = one["num_rendered"]
        r_one = one["saved"][7].to(torch.int64)
        r_grp = o["saved"][7].to(torch.int64)
        nonempty = r_one[:, 1] > r_one[:, 0]
        assert torch.equal(r_grp[nonempty] - base, r_one[nonempty])
        assert bool((r_grp[~nonempty, 1] == r_grp[~nonempty, 0]).all())
        assert torch.equal(o["saved"][8][base:base + n], one["saved"][8])
        assert torch.equal(o["out_color"], one["out_color"])
        for k in (0, 1, 2, 3, 4, 9, 10):  # radii, transforms, opacity, softness, dirs, T, last
            assert torch.equal(o["saved"][k], one["saved"][k]), k
        base += n
    assert base == outs[0]["saved"][8].numel()


def test_grouped_views_step_equals_per_view():
    """multiview.fit_step_views with the views binned in groups (of one size,
    or of the sizes given) gives the gradients and loss of the per-view step
    (to the order of the float atomics), over one and two streams."""
    import multiview
    import workloads

    w = workloads.hexels3d_tiny(13, 2000, 96, 80, 7, 0.06).to("cuda")
    params = [w.means3d, w.scales, w.rotations, w.colors, w.color_grads, w.view_grads,
              w.opacities]
    g = torch.Generator().manual_seed(6)
    cams = w.cameras
    targets = [torch.rand((3, c.height, c.width), generator=g).cuda() for c in cams]

    def step(pipe, group):
        grads = [torch.zeros_like(p) for p in params]
        loss = torch.zeros(1, device="cuda")
        multiview.fit_step_views(params, cams, targets, w.background, w.softness, grads, loss,
                                 pipe, group=group)
        torch.cuda.synchronize()
        return grads, loss

    want_g, want_l = step(None, 1)
    for pipe, group in ((None, 3), (multiview.ViewPipeline(params, streams=2), 3),
                        (multiview.ViewPipeline(params, streams=2), 7),
                        (multiview.ViewPipeline(params, streams=2), [2, 1, 4])):
        got_g, got_l = step(pipe, group)
        assert abs(float(got_l) - float(want_l)) <= 1e-5 * abs(float(want_l))
        for name, a, b in zip(multiview.PARAM_NAMES, got_g, want_g):
            assert_grad_parity(a, b, None, name)
