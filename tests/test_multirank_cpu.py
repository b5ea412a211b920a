"""Multi-rank partitioning on CPU (gloo, world size 2), computed with the
oracle: the view split of the 3D multi-view step and the tile-row stripes of
the 2D Image-GS step must give, after the all-reduce, exactly the gradients
of the single-process computation over all views / the whole image."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import sharding
import workloads

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# --------------------------------------------------------------------------
# 3D: views dealt round-robin, per-surfel gradients summed with all-reduce
# --------------------------------------------------------------------------
def _scene3d():
    return workloads.hexels3d_tiny(seed=9, num_points=120, width=40, height=32, num_views=4,
                                   scale=0.1)


def _view_grads(w, v):
    from oracle import hexels3d as o

    cam = w.cameras[v]
    g = torch.Generator().manual_seed(100 + v)
    up = {"color": torch.rand((3, cam.height * cam.width), generator=g) - 0.5}
    r = o.forward_backward(w.means3d, w.scales, w.rotations, w.opacities, w.colors,
                           w.color_grads, w.view_grads, w.background, cam, w.softness,
                           upstream=up)
    gr = r["grads"]
    return [gr["means3d"], gr["scales"], gr["rotations"], gr["colors"], gr["color_grads"],
            gr["view_grads"], gr["opacities"]]


def _params3d(w):
    return [w.means3d, w.scales, w.rotations, w.colors, w.color_grads, w.view_grads,
            w.opacities]


def _worker3d(rank, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        w = _scene3d()
        buf = sharding.GradBuffer([p.shape for p in _params3d(w)], "cpu")
        for v in sharding.view_split(len(w.cameras), WORLD, rank):
            for acc, g in zip(buf.views, _view_grads(w, v)):
                acc.add_(g.reshape(acc.shape))
            buf.loss.add_(1.0)
        buf.all_reduce_(WORLD)
        if rank == 0:
            torch.save([t.clone() for t in buf.views] + [buf.loss.clone()], out)
    finally:
        dist.destroy_process_group()


def test_view_split_partitions_views():
    for world in (1, 2, 3, 8):
        got = sorted(v for r in range(world) for v in sharding.view_split(64, world, r))
        assert got == list(range(64))
        sizes = [len(sharding.view_split(64, world, r)) for r in range(world)]
        assert max(sizes) - min(sizes) <= 1


def test_balance_views_partitions_and_balances():
    rng = np.random.default_rng(5)
    for world in (1, 2, 3, 8):
        costs = (1.0 + rng.random(64) * 3.0).tolist()
        split = sharding.balance_views(costs, world)
        assert len(split) == world
        assert sorted(v for part in split for v in part) == list(range(64))
        assert all(part == sorted(part) for part in split)
        assert split == sharding.balance_views(list(costs), world)  # deterministic
        loads = [sum(costs[v] for v in part) for part in split]
        # longest-first greedy: the heaviest rank exceeds the mean by at most one view's cost
        assert max(loads) <= sum(costs) / world + max(costs) + 1e-9
    # equal costs: a round-robin-like split, sizes within one
    sizes = [len(p) for p in sharding.balance_views([1.0] * 64, 8)]
    assert sizes == [8] * 8


def _worker_balance(rank, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        # each rank knows only the costs of its round-robin views; after the
        # all-reduce of the per-view vector every rank computes the same split
        truth = [1.0 + (7 * v % 11) for v in range(16)]
        costs = torch.zeros(16, dtype=torch.float64)
        for v in sharding.view_split(16, WORLD, rank):
            costs[v] = truth[v]
        dist.all_reduce(costs)
        split = sharding.balance_views(costs.tolist(), WORLD)
        torch.save(split, out + f".{rank}")
    finally:
        dist.destroy_process_group()


def test_balanced_split_agrees_across_ranks(tmp_path):
    out = str(tmp_path / "split")
    mp.start_processes(_worker_balance, args=(_free_port(), out), nprocs=WORLD,
                       start_method="spawn")
    s0, s1 = torch.load(out + ".0"), torch.load(out + ".1")
    assert s0 == s1
    truth = [1.0 + (7 * v % 11) for v in range(16)]
    assert s0 == sharding.balance_views(truth, WORLD)


def test_multiview_allreduce_equals_single_process(tmp_path):
    out = str(tmp_path / "grads3d.pt")
    mp.start_processes(_worker3d, args=(_free_port(), out), nprocs=WORLD, start_method="spawn")
    got = torch.load(out)
    w = _scene3d()
    want = [torch.zeros_like(p) for p in _params3d(w)]
    for v in range(len(w.cameras)):
        for acc, g in zip(want, _view_grads(w, v)):
            acc.add_(g.reshape(acc.shape))
    assert float(got[-1]) == len(w.cameras)
    for a, b in zip(got[:-1], want):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


# --------------------------------------------------------------------------
# 2D: tile-row stripes, packed per-Gaussian gradients all-reduced
# --------------------------------------------------------------------------
def _stripe_grads(w, rows):
    """Oracle fwd+bwd of the Image-GS L2 loss restricted to tile rows
    [rows[0], rows[1]) (all rows when None); returns (v_xy, v_conic,
    v_colors, image rows rendered)."""
    from oracle import raster2d as o

    tx, ty, _ = w.tile_bounds
    xys, radii, conics, _ = o.project_2d(w.means2d, w.scales2d, w.rotation, w.height, w.width,
                                         w.tile_bounds)
    r0, r1 = (0, ty) if rows is None else rows
    keys, ids = o.map_intersects(xys.numpy(), radii.numpy(), None, w.tile_bounds,
                                 tile_rows=(r0, r1))
    _, ids_sorted, bins = o.sort_and_bin(keys, ids, tx * ty)
    tiles = np.arange(r0 * tx, r1 * tx)
    img, topk, _, _ = o.rasterize_topk_forward(xys, conics, w.colors,
                                               torch.from_numpy(ids_sorted), bins, w.height,
                                               w.width, tile_ids=tiles)
    y0, y1 = r0 * 16, min(r1 * 16, w.height)
    numel = img.numel()
    v_img = torch.zeros_like(img)
    v_img[y0:y1] = 2.0 * (img[y0:y1] - w.target[y0:y1]) / numel
    topk_s = torch.full_like(topk, -1)
    topk_s[y0:y1] = topk[y0:y1]
    v_xy, v_conic, v_col = o.rasterize_topk_backward(xys, conics, w.colors, v_img, topk_s,
                                                     w.height, w.width)
    return v_xy, v_conic, v_col, img[y0:y1]


def _worker2d(rank, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        w = workloads.imagegs_tiny()
        rows = sharding.stripe_rows(w.tile_bounds[1], WORLD, rank)
        v_xy, v_conic, v_col, img = _stripe_grads(w, rows)
        buf = sharding.GradBuffer([v_xy.shape, v_conic.shape, v_col.shape], "cpu")
        for acc, g in zip(buf.views, (v_xy, v_conic, v_col)):
            acc.copy_(g)
        buf.all_reduce_(WORLD)
        torch.save({"rank": rank, "img": img, "rows": rows}, out + f".{rank}")
        if rank == 0:
            torch.save([t.clone() for t in buf.views], out)
    finally:
        dist.destroy_process_group()


def test_stripes_partition_rows():
    for ty in (1, 3, 128):
        for world in (1, 2, 4, 8):
            rows = [sharding.stripe_rows(ty, world, r) or (0, ty) for r in range(world)]
            assert rows[0][0] == 0 and rows[-1][1] == ty
            assert all(a[1] == b[0] for a, b in zip(rows[:-1], rows[1:]))


def test_stripe_allreduce_equals_full_image(tmp_path):
    out = str(tmp_path / "grads2d.pt")
    mp.start_processes(_worker2d, args=(_free_port(), out), nprocs=WORLD, start_method="spawn")
    got = torch.load(out)
    w = workloads.imagegs_tiny()
    v_xy, v_conic, v_col, img = _stripe_grads(w, None)
    for a, b in zip(got, (v_xy, v_conic, v_col)):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-7)
    # the stripes' pixels are the full image's
    parts = sorted((torch.load(out + f".{r}") for r in range(WORLD)), key=lambda d: d["rank"])
    torch.testing.assert_close(torch.cat([p["img"] for p in parts]), img, rtol=0, atol=0)
