"""The exact-sort and pixel-risk diagnostics against the reference's own
kernels (oracle/_ref): every exact_mode, a selected-surfel mask, a pixel mask,
crops, and a crop of the 1M-surfel 1080p view.

Tolerances: hit counts, enabled mask and order-changed flags bit-exact; the
recomposited image and the risk map within 1e-5 absolute.
"""

from __future__ import annotations

import pytest
import torch

from conftest import ref_module

pytestmark = pytest.mark.gpu
ATOL = 1e-5


@pytest.fixture(scope="module")
def ref():
    r = ref_module("_ref_hexels3d_C")
    if r is None:
        pytest.skip("reference kernels not built")
    return r


def _inputs(size="tiny", seed=31):
    import workloads

    if size == "tiny":
        w = workloads.hexels3d_tiny(seed, 1500, 88, 72, 2, 0.06).to("cuda")
    else:
        w = workloads.hexels3d_single().to("cuda")
    cam = w.cameras[0]
    g = torch.Generator().manual_seed(seed)
    P = w.num_points
    e = torch.empty(0, device="cuda")
    native = torch.rand((3, cam.height, cam.width), generator=g).cuda()
    selected = (torch.rand((P,), generator=g) < 0.3).cuda()
    pixel_mask = (torch.rand((cam.height, cam.width), generator=g) < 0.5).cuda()
    quads = (0.05 * torch.randn((P, 3, 3), generator=g)).cuda()
    ks = (0.2 * torch.rand((P, 3), generator=g)).cuda()
    ls = (3 * torch.rand((P,), generator=g) - 0.5).cuda()
    return w, cam, e, native, selected, pixel_mask, quads, ks, ls


def _tensors(w, cam, e, quads, ks, ls, cm, vm):
    cg = w.color_grads if cm >= 1 else e
    cq = quads if cm >= 2 else e
    vg = w.view_grads if vm == 1 else e
    return (w.means3d, w.scales, w.rotations, w.colors, cg, cq, vg,
            ks if vm == 2 else e, ls if vm == 2 else e, w.opacities, e, cam.viewmatrix,
            cam.projmatrix, cam.campos, w.background)


def _check(mine, theirs, names):
    for n, a, b in zip(names, mine, theirs):
        assert a.shape == b.shape and a.dtype == b.dtype, n
        if a.dtype.is_floating_point:
            torch.testing.assert_close(a, b, rtol=0, atol=ATOL, msg=n)
        else:
            assert torch.equal(a, b), f"{n}: {int((a != b).sum())} entries differ"


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("cm,vm", [(1, 1), (3, 2)])
def test_exact_sort_matches_reference(ref, mode, cm, vm):
    from gsplat.cuda_hexels3d import _C

    w, cam, e, native, selected, _, quads, ks, ls = _inputs()
    t = _tensors(w, cam, e, quads, ks, ls, cm, vm)
    for crop in ((0, 0, cam.width, cam.height), (13, 7, 61, 50)):
        args = (*t, native, selected, cam.width, cam.height, w.softness, 1.0, cm, vm, vm == 1,
                mode, *crop, False)
        mine = _C.rasterize_hexels3d_exact_sort_forward(*args)
        theirs = ref.rasterize_hexels3d_exact_sort_forward(*args)
        _check(mine, theirs, ("image", "order_changed", "hit_counts", "enabled"))


@pytest.mark.parametrize("cm,vm", [(1, 1), (0, 0), (2, 2)])
def test_pixel_risk_matches_reference(ref, cm, vm):
    from gsplat.cuda_hexels3d import _C

    w, cam, e, native, _, pixel_mask, quads, ks, ls = _inputs(seed=32)
    t = _tensors(w, cam, e, quads, ks, ls, cm, vm)
    for crop in ((0, 0, cam.width, cam.height), (5, 20, 80, 64)):
        args = (*t, native, pixel_mask, cam.width, cam.height, w.softness, 1.0, cm, vm, vm == 1,
                *crop, False)
        mine = _C.rasterize_hexels3d_pixel_risk_forward(*args)
        theirs = ref.rasterize_hexels3d_pixel_risk_forward(*args)
        _check(mine, theirs, ("image", "risk", "order_changed", "hit_counts", "enabled"))


def test_full_view_crop_matches_reference(ref):
    """A 256x128 crop of the 1M-surfel 1080p view: every hit's depth
    re-sort (crop_all) and the risk map."""
    from gsplat.cuda_hexels3d import _C

    w, cam, e, native, selected, pixel_mask, quads, ks, ls = _inputs("full", seed=33)
    t = _tensors(w, cam, e, quads, ks, ls, 1, 1)
    crop = (832, 476, 1088, 604)
    args = (*t, native, selected, cam.width, cam.height, w.softness, 1.0, 1, 1, True, 3, *crop,
            False)
    mine = _C.rasterize_hexels3d_exact_sort_forward(*args)
    theirs = ref.rasterize_hexels3d_exact_sort_forward(*args)
    _check(mine, theirs, ("image", "order_changed", "hit_counts", "enabled"))
    assert int(mine[1].sum()) > 0  # some pixels do reorder
    args = (*t, native, pixel_mask, cam.width, cam.height, w.softness, 1.0, 1, 1, True, *crop,
            False)
    _check(_C.rasterize_hexels3d_pixel_risk_forward(*args),
           ref.rasterize_hexels3d_pixel_risk_forward(*args),
           ("image", "risk", "order_changed", "hit_counts", "enabled"))


def test_public_wrappers_and_argument_errors():
    import gsplat

    w, cam, e, native, selected, pixel_mask, *_ = _inputs(seed=34)
    args = (w.means3d, w.scales, w.rotations, w.colors, w.color_grads, w.view_grads,
            w.opacities, cam.viewmatrix, cam.projmatrix, cam.campos, w.background, native)
    img, changed, hits, enabled = gsplat.rasterize_hexels3d_exact_sort_forward(
        *args, selected, cam.width, cam.height, w.softness, mode="hybrid",
        crop_xyxy=(0, 0, 40, 40))
    assert img.shape == native.shape and bool(enabled[40:, :].logical_not().all())
    assert torch.equal(img[:, 40:, :], native[:, 40:, :])
    out = gsplat.rasterize_hexels3d_pixel_risk_forward(*args, pixel_mask, cam.width, cam.height,
                                                       w.softness)
    assert len(out) == 5 and torch.isfinite(out[1]).all()
    with pytest.raises(ValueError, match="Unknown exact-sort mode"):
        gsplat.rasterize_hexels3d_exact_sort_forward(*args, selected, cam.width, cam.height,
                                                     w.softness, mode="nope")
    with pytest.raises(RuntimeError, match="crop must satisfy"):
        gsplat.rasterize_hexels3d_exact_sort_forward(*args, selected, cam.width, cam.height,
                                                     w.softness, crop_xyxy=(10, 0, 5, 4))
