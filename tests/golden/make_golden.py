"""Generate the golden vectors of tests/golden/ from the reference's own CUDA
kernels, compiled from its sources into oracle/_ref (oracle/build_ref.py).

Run on a CUDA machine from the repository root:

    python tests/golden/make_golden.py

Writes three small fixtures, each holding the inputs and the reference's
outputs on them:

  imagegs.pt   Image-GS 2D: projection, intersections, sorted lists and tile
               bins, top-10 normalised compositing (with the weight-sum and
               entropy statistics) and its backward, projection backward
               (48x72 image, 96 Gaussians, imagegs_tiny(seed=7)).
  hexels2d.pt  2D image hexels: forward/backward of the plain and the
               affine + colour-gradient + per-edge-softness variants
               (40x56 image, 60 hexagons, hexels2d_tiny(seed=3)).
  hexels3d.pt  3D hexel surfels: the cached forward's eleven saved buffers,
               image and cached backward; the surface forward (depth, alpha,
               normal, distortion, median) and its uncached backward
               (88x72 image, 1500 surfels, hexels3d_tiny(seed=1)).

The reference sorts intersections with torch.sort; here the sort is stable
(ties keep index order), matching the stable radix sort the B200 build uses.
"""

from __future__ import annotations

import importlib.util
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "hexel-kernel_b200"))
sys.path.insert(0, ROOT)

import workloads  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def _ref(name):
    path = os.path.join(ROOT, "oracle", "_ref", name + ".so")
    if not os.path.exists(path):
        raise SystemExit(f"{path} is missing: build it with python oracle/build_ref.py")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _cpu(d):
    out = {}
    for k, v in d.items():
        if torch.is_tensor(v):
            out[k] = v.detach().cpu().clone()
        elif isinstance(v, (list, tuple)) and v and torch.is_tensor(v[0]):
            out[k] = [t.detach().cpu().clone() for t in v]
        else:
            out[k] = v
    return out


def _bin2d(ref, n, xys, radii, nth, tb):
    cum = torch.cumsum(nth, 0, dtype=torch.int32)
    ni = int(cum[-1].item()) if n else 0
    isect, gids = ref.map_gaussian_to_intersects(n, ni, xys, radii, cum, tb)
    isect_s, order = torch.sort(isect, stable=True)
    gids_s = torch.gather(gids, 0, order)
    bins = ref.get_tile_bin_edges(ni, tb[0] * tb[1], isect_s)
    return ni, cum, isect, gids, isect_s, gids_s, bins


def imagegs(ref):
    w = workloads.imagegs_tiny(7, 48, 72, 96, 3.0)
    dev = "cuda"
    m, s, r, c = (t.to(dev) for t in (w.means2d, w.scales2d, w.rotation, w.colors))
    H, W, tb, n = w.height, w.width, w.tile_bounds, w.num_points
    xys, radii, conics, nth = ref.project_gaussians_2d_scale_rot_forward(n, m, s, r, H, W, tb)
    ni, cum, isect, gids, isect_s, gids_s, bins = _bin2d(ref, n, xys, radii, nth, tb)
    img, topk, ws, ent = ref.nd_rasterize_forward_topk_norm_stats(
        tb, (16, 16, 1), (W, H, 1), gids_s, bins, xys, conics, c)
    g = torch.Generator().manual_seed(2)
    v_out = (torch.rand(img.shape, generator=g) * 2 - 1).to(dev)
    v_ws = (0.1 * torch.randn((H, W), generator=g)).to(dev)
    v_en = (0.1 * torch.randn((H, W), generator=g)).to(dev)
    v_xy, v_conic, v_col = ref.nd_rasterize_backward_topk_norm_stats(
        H, W, 16, 16, gids_s, bins, xys, conics, c, v_out, v_ws, v_en, topk)
    pb = ref.project_gaussians_2d_scale_rot_backward(n, m, s, r, H, W, radii, conics, v_xy,
                                                     v_conic)
    return _cpu(dict(
        height=H, width=W, tile_bounds=tb, means2d=m, scales2d=s, rotation=r, colors=c,
        xys=xys, radii=radii, conics=conics, num_tiles_hit=nth, num_intersects=ni, cum=cum,
        isect_ids=isect, gaussian_ids=gids, isect_ids_sorted=isect_s, gaussian_ids_sorted=gids_s,
        tile_bins=bins, img=img, pixel_topk=topk, weights_sum=ws, entropy=ent, v_out=v_out,
        v_weights_sum=v_ws, v_entropy=v_en, v_xy=v_xy, v_conic=v_conic, v_colors=v_col,
        v_cov2d=pb[0], v_mean2d=pb[1], v_scale=pb[2], v_rot=pb[3]))


def hexels2d(ref):
    w = workloads.hexels2d_tiny(3, 40, 56, 60)
    dev = "cuda"
    n, H, W, tb = w.num_points, w.height, w.width, w.tile_bounds
    g = torch.Generator().manual_seed(3)
    xys, scales, rot, col = (t.to(dev) for t in (w.xys, w.scales, w.rotation, w.colors))
    affines = (torch.tensor([[0.3, 0.02], [-0.03, 0.28]]).repeat(n, 1, 1)
               * (0.8 + 0.4 * torch.rand((n, 1, 1), generator=g))).to(dev)
    cgr = (0.05 * torch.randn((n, 2, 3), generator=g)).to(dev)
    soft3 = (8 + 4 * torch.rand((n, 3), generator=g)).to(dev)
    sharp = (0.02 + 0.05 * torch.rand((n,), generator=g)).to(dev)
    emis = (0.1 * torch.rand((n, 3), generator=g)).to(dev)
    radii = w.radii.to(dev)
    # tiles touched per hexagon from the caller's radii, by the reference's
    # get_tile_bbox (gsplat/cuda/csrc/helpers.cuh:11-43)
    cx, cy = xys[:, 0] / 16.0, xys[:, 1] / 16.0
    rt = radii.float() / 16.0
    x0 = (cx - rt).to(torch.int32).clamp(0, tb[0])
    x1 = (cx + rt + 1).to(torch.int32).clamp(0, tb[0])
    y0 = (cy - rt).to(torch.int32).clamp(0, tb[1])
    y1 = (cy + rt + 1).to(torch.int32).clamp(0, tb[1])
    nth = torch.where(radii > 0, (x1 - x0) * (y1 - y0), torch.zeros_like(radii)).to(torch.int32)
    ni, cum, isect, gids, isect_s, gids_s, bins = _bin2d(ref, n, xys, radii, nth, tb)
    out = dict(height=H, width=W, tile_bounds=tb, softness=w.softness, xys=xys, scales=scales,
               rotation=rot, colors=col, affines=affines, color_grads=cgr, softnesses3=soft3,
               sharpness=sharp, emission=emis, radii=radii, gaussian_ids_sorted=gids_s,
               tile_bins=bins)
    aa = 0.3
    img, topk, ws, ent = ref.nd_rasterize_forward_topk_norm_hexels(
        tb, (16, 16, 1), (W, H, 1), gids_s, bins, xys, scales, rot, col, aa, w.softness, sharp,
        emis)
    g2 = torch.Generator().manual_seed(11)
    v_out = (torch.rand(img.shape, generator=g2) * 2 - 1).to(dev)
    v_ws = (0.1 * torch.randn(ws.shape, generator=g2)).to(dev)
    v_en = (0.1 * torch.randn(ent.shape, generator=g2)).to(dev)
    b = ref.nd_rasterize_backward_topk_norm_hexels(
        H, W, 16, 16, gids_s, bins, xys, scales, rot, col, v_out, v_ws, v_en, topk, aa,
        w.softness, sharp, emis)
    out.update(aa=aa, plain_img=img, plain_topk=topk, plain_ws=ws, plain_ent=ent, v_out=v_out,
               v_ws=v_ws, v_en=v_en, plain_grads=list(b))
    img, topk, ws, ent = ref.nd_rasterize_forward_topk_norm_hexels_affine_color_grad_softness(
        tb, (16, 16, 1), (W, H, 1), gids_s, bins, xys, affines, col, cgr, 0.7, aa, soft3,
        w.softness, sharp, emis)
    b = ref.nd_rasterize_backward_topk_norm_hexels_affine_color_grad_softness(
        H, W, 16, 16, gids_s, bins, xys, affines, col, cgr, soft3, 0.7, v_out, v_ws, v_en, topk,
        aa, w.softness, sharp, emis)
    out.update(full_img=img, full_topk=topk, full_ws=ws, full_ent=ent, full_grads=list(b))
    return _cpu(out)


def hexels3d(ref):
    w = workloads.hexels3d_tiny(1, 1500, 88, 72, 2, 0.06).to("cuda")
    cam = w.cameras[0]
    e = torch.empty(0, device="cuda")
    tens = (w.means3d, w.scales, w.rotations, w.colors, w.color_grads, e, w.view_grads, e, e,
            w.opacities, e, cam.viewmatrix, cam.projmatrix, cam.campos, w.background)
    scal = (cam.width, cam.height, cam.tan_fovx, cam.tan_fovy, w.softness, 1.0, 1, 1, True)
    img, radii, saved = ref.rasterize_hexels3d_forward_cached(*tens, *scal, False, False, False)
    H, W = cam.height, cam.width
    g = torch.Generator().manual_seed(7)
    gc = (torch.rand((3, H, W), generator=g) * 2 - 1).cuda()
    gd = (0.1 * (torch.rand((H, W), generator=g) * 2 - 1)).cuda()
    ga = (torch.rand((H, W), generator=g) * 2 - 1).cuda()
    gn = (torch.rand((5, H, W), generator=g) * 2 - 1).cuda()
    m2d = torch.zeros((w.num_points, 4), device="cuda")
    grads = ref.rasterize_hexels3d_backward_cached(w.means3d, m2d, *tens[1:], gc, e, e, e, e,
                                                   *scal, -1, False, False, False, list(saved))
    surf = ref.rasterize_hexels3d_forward_median(*tens, *scal, False, False, False, True, -1,
                                                 False, False, False)
    sgrads = ref.rasterize_hexels3d_backward(w.means3d, e, *tens[1:], gc, e, gd, ga, gn, *scal,
                                             -1, False, False, False)
    return _cpu(dict(
        width=W, height=H, tan_fovx=cam.tan_fovx, tan_fovy=cam.tan_fovy, softness=w.softness,
        means3d=w.means3d, scales=w.scales, rotations=w.rotations, colors=w.colors,
        color_grads=w.color_grads, view_grads=w.view_grads, opacities=w.opacities,
        background=w.background, viewmatrix=cam.viewmatrix, projmatrix=cam.projmatrix,
        campos=cam.campos, img=img, radii=radii, saved=list(saved), grad_color=gc,
        grad_depth=gd, grad_alpha=ga, grad_surface=gn, grads=list(grads),
        surf_color=surf[0], surf_depth=surf[5], surf_alpha=surf[6], surf_maps=surf[7],
        surf_grads=list(sgrads)))


def main() -> int:
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--out", default=OUT, help="output directory (default: tests/golden)")
    out = ap.parse_args().out
    if not torch.cuda.is_available():
        raise SystemExit("a CUDA GPU is needed to run the reference kernels")
    os.makedirs(out, exist_ok=True)
    r2 = _ref("_ref_gsplat_csrc")
    r3 = _ref("_ref_hexels3d_C")
    torch.save(imagegs(r2), os.path.join(out, "imagegs.pt"))
    torch.save(hexels2d(r2), os.path.join(out, "hexels2d.pt"))
    torch.save(hexels3d(r3), os.path.join(out, "hexels3d.pt"))
    for f in ("imagegs.pt", "hexels2d.pt", "hexels3d.pt"):
        print(f, os.path.getsize(os.path.join(out, f)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
