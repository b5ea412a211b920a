"""The multi-GPU paths on two GPUs with NCCL (skipped with fewer): the CUDA
kernels, the sharding helpers and the in-place all-reduce of the packed
gradient buffer, against one process doing all the work.

* 3D views: each rank runs its round-robin share of the views of one scene
  through multiview.fit_step_views into a sharding.GradBuffer, all-reduced;
  the result equals the single-process step over all views (to the order of
  the float atomics).
* Image-GS stripes: each rank renders its tile-row stripe
  (rasterize_gaussians_sum(tile_rows=)) and back-propagates it; the packed
  per-Gaussian gradients all-reduced equal the full image's.

Ranks are spawned processes (one per GPU, NCCL over 127.0.0.1, a short
process-group timeout); each writes its result for rank 0 to compare.
"""

from __future__ import annotations

import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _params_3d():
    import workloads

    w = workloads.hexels3d_tiny(21, 3000, 96, 80, 6, 0.06)
    return w, [w.means3d, w.scales, w.rotations, w.colors, w.color_grads, w.view_grads,
               w.opacities]


def _targets(w):
    g = torch.Generator().manual_seed(9)
    return [torch.rand((3, c.height, c.width), generator=g) for c in w.cameras]


def _step_3d(w, params, cams, targets, world):
    import multiview
    import sharding

    grads = sharding.GradBuffer([p.shape for p in params], "cuda")
    pipe = multiview.ViewPipeline(params, streams=2)
    multiview.fit_step_views(params, cams, targets, w.background.cuda(), w.softness,
                             grads.views, grads.loss, pipe)
    grads.all_reduce_(world)
    torch.cuda.synchronize()
    return grads.flat.cpu()


def _imagegs(tile_rows):
    import gsplat
    import workloads

    w = workloads.imagegs_tiny(seed=4, height=96, width=80, num_points=300)
    leaves = [t.cuda().clone().requires_grad_() for t in (w.means2d, w.scales2d, w.rotation,
                                                          w.colors)]
    m, s, r, c = leaves
    xys, radii, conics, nth = gsplat.project_gaussians_2d_scale_rot(m, s, r, w.height, w.width,
                                                                    w.tile_bounds)
    img = gsplat.rasterize_gaussians_sum(xys, radii, conics, nth, c, w.height, w.width,
                                         topk_norm=True, tile_rows=tile_rows)
    up = torch.rand(img.shape, generator=torch.Generator().manual_seed(2)).cuda() * 2 - 1
    (img * up).sum().backward()
    return w, torch.cat([x.grad.reshape(-1) for x in leaves])


def _worker(rank, world, port, out_dir):
    for p in (os.path.join(ROOT, "hexel-kernel_b200"), ROOT, os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    import sharding

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        w, params = _params_3d()
        params = [p.cuda() for p in params]
        cams = [w.cameras[v].to("cuda") for v in sharding.view_split(len(w.cameras), world, rank)]
        targets = _targets(w)
        mine = [targets[v].cuda() for v in sharding.view_split(len(w.cameras), world, rank)]
        flat3d = _step_3d(w, params, cams, mine, world)
        wi, _ = _imagegs(None)
        rows = sharding.stripe_rows(wi.tile_bounds[1], world, rank)
        _, g2d = _imagegs(rows)
        g2d = g2d.contiguous()
        dist.all_reduce(g2d)
        torch.cuda.synchronize()
        torch.save({"flat3d": flat3d, "g2d": g2d.cpu()}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_views_and_stripes_match_one_process(tmp_path):
    import torch.multiprocessing as mp

    from conftest import assert_grad_parity

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [torch.load(os.path.join(tmp_path, f"r{r}.pt")) for r in range(world)]
    # single process, all views / the full image, on GPU 0
    w, params = _params_3d()
    params = [p.cuda() for p in params]
    cams = [c.to("cuda") for c in w.cameras]
    want3d = _step_3d(w, params, cams, [t.cuda() for t in _targets(w)], 1)
    _, want2d = _imagegs(None)
    for r in res:
        assert_grad_parity(r["flat3d"], want3d, None, "3D views, packed gradients + loss")
        assert_grad_parity(r["g2d"], want2d, None, "Image-GS stripes, packed gradients")
    assert torch.equal(res[0]["flat3d"], res[1]["flat3d"])
