"""The oracle against golden vectors recorded from the reference's own CUDA
kernels (tests/golden/make_golden.py).  CPU only.

Integer outputs computed by the oracle from the reference's float inputs
(intersection keys, sorted lists, tile bins) must match exactly; float
outputs agree to fp32 tolerance (the CPU uses IEEE exp/division where the
reference uses fast-math intrinsics and fused multiply-adds); top-K lists
agree on all but tie-breaking pixels.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import assert_close_oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not generated (tests/golden/make_golden.py on a GPU)")
    return torch.load(path, map_location="cpu", weights_only=False)


def _close(a, b, rtol, atol_frac, name=""):
    a, b = a.double(), b.double()
    atol = atol_frac * max(1.0, float(b.abs().max()) if b.numel() else 1.0)
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol, msg=name)


def test_imagegs_golden():
    from oracle import raster2d as o

    g = _load("imagegs.pt")
    H, W, tb = g["height"], g["width"], tuple(g["tile_bounds"])
    xys, radii, conics, nth = o.project_2d(g["means2d"], g["scales2d"], g["rotation"], H, W, tb)
    torch.testing.assert_close(xys, g["xys"], rtol=1e-6, atol=1e-4)
    torch.testing.assert_close(conics, g["conics"], rtol=1e-4, atol=1e-6)
    assert (radii != g["radii"]).float().mean() < 0.02
    # binning of the reference's projection outputs: exact
    keys, ids = o.map_intersects(g["xys"].numpy(), g["radii"].numpy(), None, tb)
    assert np.array_equal(keys, g["isect_ids"].numpy())
    assert np.array_equal(ids, g["gaussian_ids"].numpy())
    ks, idss, bins = o.sort_and_bin(keys, ids, tb[0] * tb[1])
    assert np.array_equal(ks, g["isect_ids_sorted"].numpy())
    assert np.array_equal(idss, g["gaussian_ids_sorted"].numpy())
    assert np.array_equal(bins, g["tile_bins"].numpy())
    # compositing on the reference's lists
    img, topk, ws, ent = o.rasterize_topk_forward(g["xys"], g["conics"], g["colors"],
                                                  g["gaussian_ids_sorted"],
                                                  g["tile_bins"].numpy(), H, W)
    same = (topk == g["pixel_topk"]).all(-1)
    assert float(same.float().mean()) >= 0.99
    torch.testing.assert_close(img[same], g["img"][same], rtol=0, atol=1e-5)
    torch.testing.assert_close(ws[same], g["weights_sum"][same], rtol=1e-5, atol=1e-5)
    vx, vc, vcol = o.rasterize_topk_backward(g["xys"], g["conics"], g["colors"], g["v_out"],
                                             g["pixel_topk"], H, W, g["v_weights_sum"],
                                             g["v_entropy"])
    _close(vx, g["v_xy"], 1e-3, 1e-5, "v_xy")
    _close(vc, g["v_conic"], 1e-3, 1e-5, "v_conic")
    _close(vcol, g["v_colors"], 1e-3, 1e-5, "v_colors")
    pb = o.project_2d_backward(g["scales2d"], g["rotation"], H, W, g["radii"], g["conics"],
                               g["v_xy"], g["v_conic"])
    for a, name in zip(pb, ("v_cov2d", "v_mean2d", "v_scale", "v_rot")):
        _close(a.reshape(g[name].shape), g[name], 1e-3, 1e-5, name)


def test_hexels2d_golden():
    from oracle import hexels2d as oh

    g = _load("hexels2d.pt")
    H, W = g["height"], g["width"]
    ids, bins = g["gaussian_ids_sorted"], g["tile_bins"].numpy()
    for kind in ("plain", "full"):
        p = oh.HexParams(xys=g["xys"], colors=g["colors"], softness=g["softness"], aa=g["aa"])
        if kind == "plain":
            p.scales, p.rotation = g["scales"], g["rotation"]
        else:
            p.affines = g["affines"]
            p.color_grads, p.color_grad_scale = g["color_grads"], 0.7
            p.softnesses = g["softnesses3"]
        p.sharpness, p.emission = g["sharpness"], g["emission"]
        img, topk, ws, ent = oh.forward(p, ids, bins, H, W)
        same = (topk == g[f"{kind}_topk"]).all(-1)
        assert float(same.float().mean()) > 0.97, kind
        torch.testing.assert_close(img[same], g[f"{kind}_img"][same], rtol=1e-5, atol=1e-5)
        og = oh.backward(p, g["v_out"], g["v_ws"], g["v_en"], g[f"{kind}_topk"], H, W)
        names = ["v_xy"] + (["v_affines"] if kind == "full" else ["v_scale", "v_rot"])
        names += ["v_colors"] + (["v_color_grads"] if kind == "full" else [])
        names += ["v_emission", "v_sharpness"] + (["v_softnesses"] if kind == "full" else [])
        for name, ref in zip(names, g[f"{kind}_grads"]):
            if name in og:
                x = og[name]
                _close(x.reshape(ref.shape), ref, 1e-3, 1e-5, f"{kind}:{name}")


def test_hexels3d_golden():
    from oracle import hexels3d as o

    g = _load("hexels3d.pt")
    W, H = g["width"], g["height"]
    saved = g["saved"]
    pre = o.preprocess(g["means3d"], g["scales"], g["rotations"], g["opacities"],
                       g["viewmatrix"], g["projmatrix"], g["campos"], W, H, g["softness"])
    radii = saved[0].numpy()
    assert (pre["radii"] == radii).mean() >= 0.995
    live = torch.from_numpy((pre["radii"] == radii) & (radii > 0))
    torch.testing.assert_close(pre["transMats"][live], saved[1][live], rtol=1e-5, atol=1e-5)
    # compositing on the reference's sorted lists
    opre = dict(transMats=saved[1], opacities=saved[2], softnesses=saved[3], softness_stride=1,
                view_dirs=saved[4], normals=o.normals_of(g["rotations"]),
                points_xy_center=torch.zeros((radii.shape[0], 2)), W=W, H=H,
                grid=((W + 15) // 16, (H + 15) // 16))
    ranges = saved[7].numpy().astype(np.int64)
    plist = saved[8].numpy()
    r = o.render(opre, ranges, plist, g["colors"], g["background"], g["color_grads"], None,
                 g["view_grads"], upstream={"color": g["grad_color"]})
    HW = W * H
    assert_close_oracle(r["color"], g["img"].reshape(3, HW), "color")
    assert_close_oracle(r["final_T"], saved[9].reshape(HW), "final_T")
    assert float((r["last_index"] == saved[10].reshape(HW).long()).float().mean()) >= 0.999
    G = r["grads"]
    gm3, gs, gq = o.geometry_backward(g["means3d"], g["scales"], g["rotations"], g["projmatrix"],
                                      g["campos"], W, H, radii, G["transMats"], G["view_dirs"])
    ref = g["grads"]
    for name, a, b in [("means3d", gm3, ref[0]), ("scales", gs, ref[2]),
                       ("rotations", gq, ref[3]), ("colors", G["colors"], ref[4]),
                       ("color_grads", G["color_grads"], ref[5]),
                       ("view_grads", G["view_grads"], ref[7]),
                       ("opacities", G["opacities"], ref[10])]:
        _close(a.reshape(b.shape), b, 1e-3, 1e-5, name)
