"""Image-GS tile-row stripes on the GPU: the CUDA path of
`rasterize_gaussians_sum(..., tile_rows=)` that shards one large image over
ranks (sharding.stripe_rows), run stripe by stripe on one GPU.

The forward is pixel-local, so every stripe's rows must equal the full
image's bit for bit (and be zero elsewhere); the gradients of the stripes
summed must equal the full image's, to the summation-order tolerance of
conftest.assert_grad_parity (float atomics add the partial sums in another
order).  Cases: a ragged tiny image (3 stripes) and the 2048x2048 /
100,000-Gaussian configuration split as over 8 ranks.
"""

from __future__ import annotations

import pytest
import torch

from conftest import assert_grad_parity

pytestmark = pytest.mark.gpu


def _render(w, up, tile_rows=None):
    import gsplat

    leaves = [t.cuda().clone().requires_grad_() for t in (w.means2d, w.scales2d, w.rotation,
                                                          w.colors)]
    m, s, r, c = leaves
    xys, radii, conics, nth = gsplat.project_gaussians_2d_scale_rot(m, s, r, w.height, w.width,
                                                                    w.tile_bounds)
    img = gsplat.rasterize_gaussians_sum(xys, radii, conics, nth, c, w.height, w.width,
                                         topk_norm=True, tile_rows=tile_rows)
    (img * up).sum().backward()
    return img.detach(), [x.grad for x in leaves]


@pytest.mark.parametrize("kind,world", [("tiny", 3), ("large", 8)])
def test_stripes_assemble_the_full_image_and_gradients(kind, world):
    import sharding
    import workloads

    w = workloads.imagegs_tiny() if kind == "tiny" else workloads.imagegs_large()
    g = torch.Generator().manual_seed(17)
    up = (torch.rand((w.height, w.width, 3), generator=g) * 2 - 1).cuda()
    full_img, full_grads = _render(w, up)
    img_sum = torch.zeros_like(full_img)
    grad_sum = [torch.zeros_like(x) for x in full_grads]
    ty = w.tile_bounds[1]
    for rank in range(world):
        r0, r1 = sharding.stripe_rows(ty, world, rank)
        img, grads = _render(w, up, (r0, r1))
        y0, y1 = r0 * 16, min(r1 * 16, w.height)
        assert torch.equal(img[y0:y1], full_img[y0:y1]), f"stripe {rank} rows differ"
        outside = torch.ones(w.height, dtype=torch.bool, device=img.device)
        outside[y0:y1] = False
        assert float(img[outside].abs().sum()) == 0.0
        img_sum += img
        for acc, x in zip(grad_sum, grads):
            acc += x
    assert torch.equal(img_sum, full_img)
    for name, a, b in zip(("means2d", "scales2d", "rotation", "colors"), grad_sum, full_grads):
        assert_grad_parity(a, b, None, name)
