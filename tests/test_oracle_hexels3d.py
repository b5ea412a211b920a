"""CPU checks of the 3D hexel surfel oracle (oracle/hexels3d.py): a
closed-form single-surfel case, binning invariants, and float64
finite-difference checks of its backward (the exact-gradient paths; the
reference's deliberate departures apply only under the prefilter and to the
overdraw of a pixel's terminating surfel, neither of which is exercised here).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import workloads
from oracle import hexels3d as o


def _single_surfel(opacity=0.8, softness=10.0, size=65, focal=64.0, scale=0.1):
    cam = workloads.look_at_camera((0.0, 0.0, 3.0), size, size, focal, focal)
    one = lambda *v: torch.tensor([list(v)], dtype=torch.float32)  # noqa: E731
    return dict(means3d=one(0.0, 0.0, 0.0), scales=one(scale, scale),
                rotations=one(1.0, 0.0, 0.0, 0.0), opacities=torch.tensor([opacity]),
                colors=one(0.9, 0.5, 0.1), color_grads=torch.zeros((1, 2, 3)),
                view_grads=torch.zeros((1, 3, 3)), background=torch.tensor([0.1, 0.2, 0.3]),
                cam=cam, softness=softness)


def test_single_surfel_closed_form():
    """A surfel at the origin facing a camera at distance 3: T's depth row is
    (0, 0, 3); along the centre row u = (px - c) * 3 / (f * s) and v = 0, so
    alpha = min(o * sigmoid(-(sqrt(3)/2 |u| - 1) k), 0.99); depth = 3; the
    rendered normal faces the camera."""
    s = _single_surfel()
    cam = s["cam"]
    r = o.forward_backward(s["means3d"], s["scales"], s["rotations"], s["opacities"], s["colors"],
                           s["color_grads"], s["view_grads"], s["background"], cam,
                           s["softness"], surface=True)
    T = r["pre"]["transMats"][0]
    torch.testing.assert_close(T[6:9], torch.tensor([0.0, 0.0, 3.0]), atol=1e-5, rtol=0)
    W = cam.width
    c = (W - 1) // 2
    for px in range(c - 4, c + 5):
        u = (px - c) * 3.0 / (64.0 * 0.1)
        dist = max(0.0, (math.sqrt(3.0) / 2.0) * abs(u)) - 1.0
        alpha = min(0.8 / (1.0 + math.exp(dist * 10.0)), 0.99)
        pix = c * W + px
        if alpha < 1.0 / 255.0:
            continue
        for ch in range(3):
            want = alpha * float(s["colors"][0, ch]) + (1 - alpha) * float(s["background"][ch])
            assert abs(float(r["color"][ch, pix]) - want) < 2e-6, (px, ch)
        assert abs(float(r["alpha"][pix]) - alpha) < 2e-6
        assert abs(float(r["depth"][pix]) - 3.0 * alpha) < 1e-5
        torch.testing.assert_close(r["normal"][:, pix], torch.tensor([0.0, 0.0, alpha]),
                                   atol=2e-6, rtol=0)


def test_binning_invariants():
    w = workloads.hexels3d_tiny(2, 800, 72, 56, 1, 0.08)
    cam = w.cameras[0]
    pre = o.preprocess(w.means3d, w.scales, w.rotations, w.opacities, cam.viewmatrix,
                       cam.projmatrix, cam.campos, cam.width, cam.height, w.softness)
    keys, ids, ranges = o.bin_surfels(pre)
    assert keys.size == int(pre["tiles_touched"].sum()) > 0
    assert np.all(keys[1:] >= keys[:-1])
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    for t in range(ranges.shape[0]):
        b, e = ranges[t]
        assert np.all(tiles[b:e] == t)
    assert int((ranges[:, 1] - ranges[:, 0]).sum()) == keys.size
    # stable: equal keys keep surfel order
    same = keys[1:] == keys[:-1]
    assert np.all(ids[1:][same] > ids[:-1][same])
    # a surfel with radius 0 touches no tile (the converse does not hold: the
    # reference keeps the radius of surfels culled by its later tests)
    assert np.all(pre["tiles_touched"][pre["radii"] == 0] == 0)


def _fd_scene(view_model=1, color_model=1):
    w = workloads.hexels3d_tiny(5, 40, 40, 32, 1, 0.12)
    g = torch.Generator().manual_seed(11)
    P = w.num_points
    extra = dict(color_quads=0.1 * torch.randn((P, 3, 3), generator=g),
                 specular_ks=0.3 * torch.rand((P, 3), generator=g),
                 specular_log_s=0.5 + 3 * torch.rand((P,), generator=g))
    return w, extra


def _loss_and_grads(w, extra, up, view_model, color_model, params=None):
    cam = w.cameras[0]
    p = dict(means3d=w.means3d, scales=w.scales, rotations=w.rotations, opacities=w.opacities,
             colors=w.colors, color_grads=w.color_grads, view_grads=w.view_grads, **extra)
    if params:
        p.update(params)
    r = o.forward_backward(p["means3d"], p["scales"], p["rotations"], p["opacities"], p["colors"],
                           p["color_grads"], p["view_grads"] if view_model == 1 else None,
                           w.background, cam, w.softness, upstream=up, surface=True,
                           color_quads=p["color_quads"] if color_model >= 2 else None,
                           specular_ks=p["specular_ks"] if view_model == 2 else None,
                           specular_log_s=p["specular_log_s"] if view_model == 2 else None,
                           color_model=color_model, view_model=view_model,
                           use_view_grads=view_model == 1)
    HW = cam.width * cam.height
    loss = (up["color"].reshape(3, HW) * r["color"]).sum()
    for k in ("depth", "alpha", "distortion"):
        loss = loss + (up[k].reshape(HW) * r[k]).sum()
    loss = loss + (up["normal"].reshape(3, HW) * r["normal"]).sum()
    return float(loss), r["grads"]


@pytest.mark.parametrize("view_model,color_model", [(1, 1), (2, 3)])
def test_backward_matches_finite_differences(view_model, color_model):
    o.set_precision(torch.float64)
    try:
        w, extra = _fd_scene()
        cam = w.cameras[0]
        HW = cam.width * cam.height
        g = torch.Generator().manual_seed(3)
        up = {"color": torch.rand((3, HW), generator=g, dtype=torch.float64) - 0.5,
              "depth": 0.05 * (torch.rand(HW, generator=g, dtype=torch.float64) - 0.5),
              "alpha": torch.rand(HW, generator=g, dtype=torch.float64) - 0.5,
              "normal": torch.rand((3, HW), generator=g, dtype=torch.float64) - 0.5,
              "distortion": torch.rand(HW, generator=g, dtype=torch.float64) - 0.5}
        base = {k: getattr(w, k).double() for k in ("means3d", "scales", "rotations", "opacities",
                                                     "colors", "color_grads", "view_grads")}
        base.update({k: v.double() for k, v in extra.items()})
        _, grads = _loss_and_grads(w, {k: base[k] for k in extra}, up, view_model, color_model,
                                   base)
        names = ["means3d", "scales", "rotations", "opacities", "colors", "color_grads"]
        names += ["view_grads"] if view_model == 1 else ["specular_ks", "specular_log_s"]
        if color_model >= 2:
            names.append("color_quads")
        # the surfels that cover the most pixels
        live = np.argsort(-np.asarray(o.preprocess(
            w.means3d, w.scales, w.rotations, w.opacities, cam.viewmatrix, cam.projmatrix,
            cam.campos, cam.width, cam.height, w.softness)["tiles_touched"]))[:4]
        eps = 1e-6
        checked = bad = 0
        for name in names:
            t = base[name]
            gt = grads[name]
            for i in live:
                for j in range(min(3, t[i].numel())):
                    pp = t.clone()
                    pm = t.clone()
                    pp.view(t.shape[0], -1)[i, j] += eps
                    pm.view(t.shape[0], -1)[i, j] -= eps
                    lp, _ = _loss_and_grads(w, {}, up, view_model, color_model,
                                            {**base, name: pp})
                    lm, _ = _loss_and_grads(w, {}, up, view_model, color_model,
                                            {**base, name: pm})
                    fd = (lp - lm) / (2 * eps)
                    an = float(gt.reshape(t.shape[0], -1)[i, j])
                    checked += 1
                    if abs(fd - an) > 1e-5 * max(1.0, abs(fd)):
                        bad += 1
        assert checked > 40
        assert bad <= checked // 20, f"{bad}/{checked} finite-difference mismatches"
    finally:
        o.set_precision(torch.float32)
