"""CPU checks of the Image-GS oracle itself (no GPU): known answers written
out by hand from the reference formulas, an independent scalar re-implementation
of the top-K insertion rule, brute-force binning, and float64
finite-difference checks of the backward passes."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import raster2d as o


@pytest.fixture
def fp64():
    o.set_precision(torch.float64)
    yield
    o.set_precision(torch.float32)


def test_known_answer_single_gaussian():
    # one Gaussian, one 16x16 tile; pixel (i=7, j=10)
    xys = torch.tensor([[10.3, 7.6]])
    conics = torch.tensor([[0.1, 0.02, 0.2]])
    colors = torch.tensor([[0.25, 0.5, 1.0]])
    ids = torch.tensor([0], dtype=torch.int32)
    bins = np.array([[0, 1]], dtype=np.int32)
    img, topk, ws, en = o.rasterize_topk_forward(xys, conics, colors, ids, bins, 16, 16)
    dx, dy = 10.3 - 10.0, 7.6 - 7.0
    sigma = 0.5 * (0.1 * dx * dx + 0.2 * dy * dy) + 0.02 * dx * dy
    alpha = math.exp(-sigma)
    denom = alpha + 1e-4
    assert abs(float(ws[7, 10]) - denom) < 1e-6
    for c in range(3):
        assert abs(float(img[7, 10, c]) - colors[0, c].item() * alpha / denom) < 1e-6
    assert topk[7, 10, 0] == 0 and (topk[7, 10, 1:] == -1).all()
    p = alpha / denom
    assert abs(float(en[7, 10]) - (-p * math.log(p + 1e-7))) < 1e-6


def _scalar_topk(alphas):
    """Independent loop form of forward.cu:255-280."""
    ids = [-1] * 10
    vals = [0.0] * 10
    for g, a in enumerate(alphas):
        mid, mval = -1, 1e30
        for k in range(10):
            if ids[k] < 0:
                mid, mval = k, -1.0
                break
            if vals[k] < mval:
                mid, mval = k, vals[k]
        if a > mval:
            ids[mid] = g
            vals[mid] = a
    return ids


def test_topk_rule_matches_scalar_loop():
    rng = np.random.default_rng(0)
    for trial in range(20):
        n = int(rng.integers(1, 40))
        alphas = rng.random(n).astype(np.float32)
        if trial % 3 == 0:  # ties
            alphas = np.round(alphas * 4) / 4
        expected = _scalar_topk(alphas.tolist())
        cands = [(torch.tensor([g]), torch.tensor([a])) for g, a in enumerate(alphas)]
        ids, _ = o._topk_select(iter(cands), 1)
        assert ids[0].tolist() == expected


def test_binning_matches_bruteforce():
    rng = np.random.default_rng(1)
    n, W, H = 60, 100, 70
    xys = (rng.random((n, 2)) * [W, H]).astype(np.float32)
    radii = rng.integers(0, 30, n).astype(np.int32)
    tb = ((W + 15) // 16, (H + 15) // 16, 1)
    keys, ids = o.map_intersects(xys, radii, None, tb)
    exp_k, exp_i = [], []
    for g in range(n):
        if radii[g] <= 0:
            continue
        cx, cy, r = xys[g, 0] / 16, xys[g, 1] / 16, radii[g] / 16
        x0 = min(max(0, int(np.float32(cx - r))), tb[0])
        x1 = min(max(0, int(np.float32(np.float32(cx + r) + 1))), tb[0])
        y0 = min(max(0, int(np.float32(cy - r))), tb[1])
        y1 = min(max(0, int(np.float32(np.float32(cy + r) + 1))), tb[1])
        for ty in range(y0, y1):
            for tx in range(x0, x1):
                exp_k.append((ty * tb[0] + tx) << 32)
                exp_i.append(g)
    assert keys.tolist() == exp_k and ids.tolist() == exp_i
    ks, is_, bins = o.sort_and_bin(keys, ids, tb[0] * tb[1])
    for t in range(tb[0] * tb[1]):
        a, b = bins[t]
        sel = [i for k, i in zip(exp_k, exp_i) if (k >> 32) == t]
        assert is_[a:b].tolist() == sel


def _tiny_scene(seed=0, n=12, H=20, W=24):
    g = torch.Generator().manual_seed(seed)
    xys = torch.rand((n, 2), generator=g, dtype=torch.float64) * torch.tensor([W, H])
    a = torch.rand(n, generator=g, dtype=torch.float64) * 0.2 + 0.05
    c = torch.rand(n, generator=g, dtype=torch.float64) * 0.2 + 0.05
    b = (torch.rand(n, generator=g, dtype=torch.float64) - 0.5) * 0.05
    conics = torch.stack([a, b, c], 1)
    colors = torch.rand((n, 3), generator=g, dtype=torch.float64)
    return xys, conics, colors


def test_topk_backward_finite_difference(fp64):
    H, W = 20, 24
    xys, conics, colors = _tiny_scene()
    tb = ((W + 15) // 16, (H + 15) // 16, 1)
    n = xys.shape[0]
    radii = np.full(n, 40, dtype=np.int32)
    keys, ids = o.map_intersects(xys.numpy().astype(np.float32), radii, None, tb)
    _, ids_s, bins = o.sort_and_bin(keys, ids, tb[0] * tb[1])
    ids_s = torch.from_numpy(ids_s)
    img, topk, _, _ = o.rasterize_topk_forward(xys, conics, colors, ids_s, bins, H, W)
    v_out = torch.rand(img.shape, generator=torch.Generator().manual_seed(9), dtype=torch.float64)
    v_xy, v_conic, v_colors = o.rasterize_topk_backward(xys, conics, colors, v_out, topk, H, W)

    def loss(x, cn, cl):
        im, tk, _, _ = o.rasterize_topk_forward(x, cn, cl, ids_s, bins, H, W)
        assert torch.equal(tk, topk)  # selection must not change under the perturbation
        return float((im * v_out).sum())

    h = 1e-6
    for (tensor, grad) in ((xys, v_xy), (conics, v_conic), (colors, v_colors)):
        for idx in [(0, 0), (3, 1), (7, 0), (n - 1, tensor.shape[1] - 1)]:
            plus = tensor.clone()
            plus[idx] += h
            minus = tensor.clone()
            minus[idx] -= h
            args_p = [xys, conics, colors]
            args_m = [xys, conics, colors]
            k = [xys is tensor, conics is tensor, colors is tensor].index(True)
            args_p[k], args_m[k] = plus, minus
            fd = (loss(*args_p) - loss(*args_m)) / (2 * h)
            assert abs(fd - float(grad[idx])) <= 1e-5 * max(1.0, abs(fd)), (idx, fd, grad[idx])


def test_projection_backward_finite_difference(fp64):
    g = torch.Generator().manual_seed(4)
    n, H, W = 8, 64, 64
    means = torch.rand((n, 2), generator=g, dtype=torch.float64)
    scales = torch.rand((n, 2), generator=g, dtype=torch.float64) * 3 + 1
    rot = torch.rand((n, 1), generator=g, dtype=torch.float64) * 6
    tb = (4, 4, 1)
    xys, radii, conics, _ = o.project_2d(means, scales, rot, H, W, tb)
    v_xy = torch.randn((n, 2), generator=g, dtype=torch.float64)
    v_conic = torch.randn((n, 3), generator=g, dtype=torch.float64)
    v_cov2d, v_mean, v_scale, v_rot = o.project_2d_backward(scales, rot, H, W, radii, conics,
                                                            v_xy, v_conic)

    # The reference's VJP (backward2d.cu:72-97) is not the exact gradient of a
    # scalar: it builds G = [[va, vb], [vb, vc]] (off-diagonal counted in both
    # entries), sums both off-diagonals of -X G X into v_cov2d.y and then
    # weights that sum by 2 again.  It equals the gradient of
    #   L(s) = va*a + 2*vb*b + vc*c   (conic (a, b, c))
    # plus v_cov2d.y * d(Sigma_01)/ds.  Both pieces are checked by FD here.
    def L(s, r):
        _, _, cn, _ = o.project_2d(means, s, r, H, W, tb)
        return (cn[:, 0] * v_conic[:, 0] + 2 * cn[:, 1] * v_conic[:, 1]
                + cn[:, 2] * v_conic[:, 2])

    def sigma01(s, r):
        R = o._rot2(r.reshape(-1))
        M = o._mat2_mul(R, o._scale2(s))
        return o._mat2_mul(M, o._t(M))[:, 0, 1]

    h = 1e-6
    for i in range(n):
        for j in range(2):
            sp, sm = scales.clone(), scales.clone()
            sp[i, j] += h
            sm[i, j] -= h
            fd = float((L(sp, rot) - L(sm, rot))[i]) / (2 * h)
            ds01 = float((sigma01(sp, rot) - sigma01(sm, rot))[i]) / (2 * h)
            expect = fd + float(v_cov2d[i, 1]) * ds01
            assert abs(expect - float(v_scale[i, j])) <= 1e-4 * max(1.0, abs(expect)), (i, j)
        rp, rm = rot.clone(), rot.clone()
        rp[i, 0] += h
        rm[i, 0] -= h
        fd = float((L(scales, rp) - L(scales, rm))[i]) / (2 * h)
        ds01 = float((sigma01(scales, rp) - sigma01(scales, rm))[i]) / (2 * h)
        expect = fd + float(v_cov2d[i, 1]) * ds01
        assert abs(expect - float(v_rot[i, 0])) <= 1e-4 * max(1.0, abs(expect)), i
    assert torch.allclose(v_mean, v_xy * torch.tensor([W, H], dtype=torch.float64))
