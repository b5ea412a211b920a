"""This build against golden vectors recorded from the reference's own CUDA
kernels (tests/golden/make_golden.py), on the GPU, without needing the
reference build: integer outputs bit-exact, images 1e-5 absolute, gradients
by conftest.assert_grad_parity."""

from __future__ import annotations

import os

import pytest
import torch

from conftest import assert_grad_parity

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not generated (tests/golden/make_golden.py on a GPU)")
    g = torch.load(path, map_location="cpu", weights_only=False)
    out = {}
    for k, v in g.items():
        if torch.is_tensor(v):
            out[k] = v.cuda()
        elif isinstance(v, list) and v and torch.is_tensor(v[0]):
            out[k] = [t.cuda() for t in v]
        else:
            out[k] = v
    return out


def test_imagegs_golden_gpu():
    from gsplat import csrc
    from gsplat.utils import bin_and_sort_gaussians

    g = _load("imagegs.pt")
    H, W, tb, n = g["height"], g["width"], tuple(g["tile_bounds"]), g["means2d"].shape[0]
    xys, radii, conics, nth = csrc.project_gaussians_2d_scale_rot_forward(
        n, g["means2d"], g["scales2d"], g["rotation"], H, W, tb)
    assert torch.equal(radii, g["radii"]) and torch.equal(nth, g["num_tiles_hit"])
    assert torch.equal(xys, g["xys"]) and torch.equal(conics, g["conics"])
    isect, gids, isect_s, gids_s, bins = bin_and_sort_gaussians(n, g["num_intersects"], xys,
                                                                radii, g["cum"], tb)
    assert torch.equal(isect, g["isect_ids"]) and torch.equal(gids, g["gaussian_ids"])
    assert torch.equal(isect_s, g["isect_ids_sorted"])
    assert torch.equal(gids_s, g["gaussian_ids_sorted"])
    assert torch.equal(bins, g["tile_bins"])
    img, topk, ws, ent = csrc.nd_rasterize_forward_topk_norm_stats(
        tb, (16, 16, 1), (W, H, 1), gids_s, bins, xys, conics, g["colors"])
    assert torch.equal(topk, g["pixel_topk"])
    for a, b in ((img, g["img"]), (ws, g["weights_sum"]), (ent, g["entropy"])):
        torch.testing.assert_close(a, b, rtol=0, atol=1e-5)
    out = csrc.nd_rasterize_backward_topk_norm_stats(
        H, W, 16, 16, gids_s, bins, xys, conics, g["colors"], g["v_out"], g["v_weights_sum"],
        g["v_entropy"], topk)
    for name, a in zip(("v_xy", "v_conic", "v_colors"), out):
        assert_grad_parity(a, g[name], None, name)
    pb = csrc.project_gaussians_2d_scale_rot_backward(n, g["means2d"], g["scales2d"],
                                                      g["rotation"], H, W, radii, conics,
                                                      g["v_xy"], g["v_conic"])
    for name, a in zip(("v_cov2d", "v_mean2d", "v_scale", "v_rot"), pb):
        assert_grad_parity(a, g[name], None, name)


def test_hexels2d_golden_gpu():
    from gsplat import csrc

    g = _load("hexels2d.pt")
    H, W, tb = g["height"], g["width"], tuple(g["tile_bounds"])
    ids, bins, aa, soft = g["gaussian_ids_sorted"], g["tile_bins"], g["aa"], g["softness"]
    img, topk, ws, ent = csrc.nd_rasterize_forward_topk_norm_hexels(
        tb, (16, 16, 1), (W, H, 1), ids, bins, g["xys"], g["scales"], g["rotation"], g["colors"],
        aa, soft, g["sharpness"], g["emission"])
    assert torch.equal(topk, g["plain_topk"])
    for a, b in ((img, g["plain_img"]), (ws, g["plain_ws"]), (ent, g["plain_ent"])):
        torch.testing.assert_close(a, b, rtol=0, atol=1e-5)
    b = csrc.nd_rasterize_backward_topk_norm_hexels(
        H, W, 16, 16, ids, bins, g["xys"], g["scales"], g["rotation"], g["colors"], g["v_out"],
        g["v_ws"], g["v_en"], topk, aa, soft, g["sharpness"], g["emission"])
    for i, (a, r) in enumerate(zip(b, g["plain_grads"])):
        assert_grad_parity(a, r, None, f"plain[{i}]")
    img, topk, ws, ent = csrc.nd_rasterize_forward_topk_norm_hexels_affine_color_grad_softness(
        tb, (16, 16, 1), (W, H, 1), ids, bins, g["xys"], g["affines"], g["colors"],
        g["color_grads"], 0.7, aa, g["softnesses3"], soft, g["sharpness"], g["emission"])
    assert torch.equal(topk, g["full_topk"])
    for a, r in ((img, g["full_img"]), (ws, g["full_ws"]), (ent, g["full_ent"])):
        torch.testing.assert_close(a, r, rtol=0, atol=1e-5)
    b = csrc.nd_rasterize_backward_topk_norm_hexels_affine_color_grad_softness(
        H, W, 16, 16, ids, bins, g["xys"], g["affines"], g["colors"], g["color_grads"],
        g["softnesses3"], 0.7, g["v_out"], g["v_ws"], g["v_en"], topk, aa, soft, g["sharpness"],
        g["emission"])
    for i, (a, r) in enumerate(zip(b, g["full_grads"])):
        assert_grad_parity(a, r, None, f"full[{i}]")


def test_hexels3d_golden_gpu():
    from gsplat.cuda_hexels3d import _C

    g = _load("hexels3d.pt")
    e = torch.empty(0, device="cuda")
    tens = (g["means3d"], g["scales"], g["rotations"], g["colors"], g["color_grads"], e,
            g["view_grads"], e, e, g["opacities"], e, g["viewmatrix"], g["projmatrix"],
            g["campos"], g["background"])
    scal = (g["width"], g["height"], g["tan_fovx"], g["tan_fovy"], g["softness"], 1.0, 1, 1, True)
    img, radii, saved = _C.rasterize_hexels3d_forward_cached(*tens, *scal, False, False, False)
    names = ["radii", "transMats", "opacities", "softnesses", "view_dirs", "normals",
             "points_xy_center", "ranges", "point_list", "final_T", "last_index"]
    for n, a, b in zip(names, saved, g["saved"]):
        if n == "final_T":
            torch.testing.assert_close(a, b, rtol=0, atol=1e-5, msg=n)
        else:
            assert a.shape == b.shape and torch.equal(a, b), n
    torch.testing.assert_close(img, g["img"], rtol=0, atol=1e-5)
    m2d = torch.zeros((g["means3d"].shape[0], 4), device="cuda")
    grads = _C.rasterize_hexels3d_backward_cached(g["means3d"], m2d, *tens[1:], g["grad_color"],
                                                  e, e, e, e, *scal, -1, False, False, False,
                                                  list(saved))
    for i, (a, b) in enumerate(zip(grads, g["grads"])):
        assert_grad_parity(a, b, None, f"grads[{i}]")
    surf = _C.rasterize_hexels3d_forward_median(*tens, *scal, False, False, False, True, -1,
                                                False, False, False)
    for a, b, n in ((surf[0], g["surf_color"], "color"), (surf[5], g["surf_depth"], "depth"),
                    (surf[6], g["surf_alpha"], "alpha"), (surf[7], g["surf_maps"], "maps")):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5 * max(1.0, float(b.abs().max())),
                                   msg=n)
    sg = _C.rasterize_hexels3d_backward(g["means3d"], e, *tens[1:], g["grad_color"], e,
                                        g["grad_depth"], g["grad_alpha"], g["grad_surface"],
                                        *scal, -1, False, False, False)
    for i, (a, b) in enumerate(zip(sg, g["surf_grads"])):
        assert_grad_parity(a, b, None, f"surf_grads[{i}]")
