"""CPU checks of the 2D-hexel oracle: known answer of the hexagon SDF, and
float64 finite-difference checks of every gradient of its backward pass."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import hexels2d as h
from oracle import raster2d as r2


@pytest.fixture
def fp64():
    r2.set_precision(torch.float64)
    yield
    r2.set_precision(torch.float32)


def test_hex_sdf_known_answers():
    u = torch.tensor([0.0, 0.0, 1.0, 0.5, 2 / math.sqrt(3), 0.0])
    v = torch.tensor([0.0, 1.0, 0.0, 0.5, 0.0, -2.0])
    dist, edge, _, _ = h.hex_sdf(u, v)
    a = float(h.HA)
    exp = [-1.0, 0.0, a - 1.0, max(0.5, a * 0.5 + 0.25, abs(a * 0.5 - 0.25)) - 1.0,
           a * 2 / math.sqrt(3) - 1.0, 1.0]
    assert torch.allclose(dist, torch.tensor(exp), atol=1e-6)
    # ties: |t2| >= |t1| picks edge 2; |v| must be strictly larger to pick 0
    assert edge[0].item() == 2 and edge[1].item() == 0 and edge[5].item() == 0


def _scene(kind: str, seed=0, n=10, H=20, W=24, C=3):
    g = torch.Generator().manual_seed(seed)
    f = torch.float64
    xys = torch.rand((n, 2), generator=g, dtype=f) * torch.tensor([W, H], dtype=f)
    colors = torch.rand((n, C), generator=g, dtype=f)
    p = h.HexParams(xys=xys, colors=colors, softness=3.0)
    if kind.startswith("affine"):
        base = torch.rand((n, 2, 2), generator=g, dtype=f) * 0.2 - 0.1
        base[:, 0, 0] += 0.25
        base[:, 1, 1] += 0.25
        p.affines = base
    else:
        p.scales = torch.rand((n, 2), generator=g, dtype=f) * 3 + 3
        p.rotation = torch.rand((n, 1), generator=g, dtype=f) * 1.0
    p.aa = 0.3
    p.softnesses = torch.rand((n, 3), generator=g, dtype=f) * 2 + 2
    p.sharpness = torch.rand((n,), generator=g, dtype=f) * 0.2 + 0.05
    p.emission = torch.rand((n, C), generator=g, dtype=f) * 0.1
    if "cgrad" in kind:
        p.color_grads = torch.randn((n, 2, C), generator=g, dtype=f) * 0.05
        p.color_grad_scale = 0.5
    return p


@pytest.mark.parametrize("kind", ["scalerot", "scalerot_cgrad", "affine", "affine_cgrad"])
def test_hexel_backward_finite_difference(fp64, kind):
    H, W = 20, 24
    p = _scene(kind)
    n = p.xys.shape[0]
    tb = ((W + 15) // 16, (H + 15) // 16, 1)
    keys, ids = r2.map_intersects(p.xys.numpy().astype(np.float32), np.full(n, 60, np.int32),
                                  None, tb)
    _, ids_s, bins = r2.sort_and_bin(keys, ids, tb[0] * tb[1])
    img, topk, ws, ent = h.forward(p, torch.from_numpy(ids_s), bins, H, W)
    gen = torch.Generator().manual_seed(5)
    v_out = torch.rand(img.shape, generator=gen, dtype=torch.float64)
    v_ws = torch.rand(ws.shape, generator=gen, dtype=torch.float64) * 0.1
    # The entropy term is left out: the reference differentiates
    # H = -sum p log(p + 1e-7) with dH/dp = -(log(p + 1e-7) + 1), dropping the
    # factor p / (p + 1e-7) (hexels_backward.cu:212-226), so its gradient is
    # not the exact derivative of the entropy it outputs.
    grads = h.backward(p, v_out, v_ws, None, topk, H, W)

    def loss(q):
        im, tk, w_, e_ = h.forward(q, torch.from_numpy(ids_s), bins, H, W)
        assert torch.equal(tk, topk)
        return float((im * v_out).sum() + (w_ * v_ws).sum())

    fields = {"v_xy": "xys", "v_colors": "colors", "v_emission": "emission",
              "v_sharpness": "sharpness", "v_softnesses": "softnesses"}
    if p.affines is not None:
        fields["v_affines"] = "affines"
    else:
        fields.update({"v_scale": "scales", "v_rot": "rotation"})
    if p.color_grads is not None:
        fields["v_color_grads"] = "color_grads"
    eps = 1e-6
    for gname, attr in fields.items():
        t = getattr(p, attr)
        gt = grads[gname].reshape(t.shape)
        flat = t.reshape(-1)
        for idx in (0, 3, flat.numel() // 2, flat.numel() - 1):
            orig = flat[idx].item()
            flat[idx] = orig + eps
            lp = loss(p)
            flat[idx] = orig - eps
            lm = loss(p)
            flat[idx] = orig
            fd = (lp - lm) / (2 * eps)
            got = float(gt.reshape(-1)[idx])
            assert abs(fd - got) <= 1e-6 * max(1.0, abs(fd)), (gname, idx, fd, got)
