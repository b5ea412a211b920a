"""GPU parity of the 3D hexel surfel rasteriser against the reference's own
CUDA kernels (oracle/_ref/_ref_hexels3d_C, compiled from its sources) and the
CPU oracle.

Tolerances: radii, transforms, tile ranges and sorted surfel lists
bit-exact; images and per-pixel outputs 1e-5 absolute; gradients per
conftest.assert_grad_parity (1e-4 relative with a 1e-5 x max|grad| floor).
"""

from __future__ import annotations

import pytest
import torch

from conftest import assert_grad_parity, ref_module

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
