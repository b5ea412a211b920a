"""Binning utilities — same API as the reference's gsplat/utils.py:12-162.

Every step runs as sm_100a kernels of ``libhexel_b200.so``: the prefix sum
replaces ``torch.cumsum``, and the stable radix sort replaces ``torch.sort`` +
``torch.gather`` (gsplat/utils.py:113,159-160).  The sorted lists are
identical to the reference's: keys ascending, and within a tile Gaussians in
ascending id order.
"""

from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor

import gsplat.cuda as _C
from ._lib import lib, ptr, stream, workspace


def map_gaussian_to_intersects(
    num_points: int,
    num_intersects: int,
    xys: Tensor,
    radii: Tensor,
    cum_tiles_hit: Tensor,
    tile_bounds: Tuple[int, int, int],
) -> Tuple[Tensor, Tensor]:
    """Map each Gaussian/tile intersection to a (tile << 32 | 0) key and the
    Gaussian's id.  Not differentiable."""
    return _C.map_gaussian_to_intersects(
        num_points, num_intersects, xys.contiguous(), radii.contiguous(),
        cum_tiles_hit.contiguous(), tile_bounds,
    )


def get_tile_bin_edges(num_intersects: int, num_tiles: int, isect_ids_sorted: Tensor) -> Tensor:
    """[start, end) of each tile's run in the sorted intersection list."""
    return _C.get_tile_bin_edges(num_intersects, num_tiles, isect_ids_sorted.contiguous())


def compute_cov2d_bounds(cov2d: Tensor) -> Tuple[Tensor, Tensor]:
    """Conic and 3-sigma radius of 2D covariances given as (N, 3) upper triangles."""
    assert cov2d.shape[-1] == 3, (
        "Expected input cov2d to be of shape (*batch, 3) (upper triangular values), "
        f"but got {tuple(cov2d.shape)}"
    )
    num_pts = cov2d.shape[0]
    assert num_pts > 0
    return _C.compute_cov2d_bounds(num_pts, cov2d.contiguous())


def _inclusive_scan(values: Tensor) -> Tuple[int, Tensor]:
    values = values.contiguous().to(torch.int32)
    dev = values.device
    n = values.numel()
    out = torch.empty((n,), dtype=torch.int32, device=dev)
    total = torch.zeros((1,), dtype=torch.int64, device=dev)
    ws = workspace(lib.query("hx_scan_workspace_bytes", n), dev)
    with torch.cuda.device(dev):
        lib.call("hx_inclusive_scan_i32", ptr(values), ptr(out), n, ptr(total), ptr(ws),
                 ws.numel(), stream(dev))
    num = int(total.item())
    if num > 2**31 - 1:
        raise RuntimeError(f"number of tile intersections {num} does not fit in int32")
    return num, out


def compute_cumulative_intersects(num_tiles_hit: Tensor) -> Tuple[int, Tensor]:
    """Inclusive prefix sum of per-Gaussian tile counts and its total
    (the total is read back to the host, as in the reference)."""
    if not num_tiles_hit.is_cuda:
        raise RuntimeError("num_tiles_hit must be a CUDA tensor")
    return _inclusive_scan(num_tiles_hit)


def sort_intersections(isect_ids: Tensor, gaussian_ids: Tensor, num_tiles: int
                       ) -> Tuple[Tensor, Tensor]:
    """Stable sort of (tile << 32 | depth-id) keys with their Gaussian ids.

    The low 32 key bits are sorted too unless they are all zero (always the
    case for keys written by map_gaussian_to_intersects)."""
    n = isect_ids.numel()
    dev = isect_ids.device
    keys_out = torch.empty_like(isect_ids)
    vals_out = torch.empty_like(gaussian_ids, dtype=torch.int32)
    if n == 0:
        return keys_out, vals_out
    tile_bits = max(1, int(num_tiles - 1).bit_length())
    low_zero = not bool(torch.any(isect_ids & 0xFFFFFFFF))
    begin = 32 if low_zero else 0
    keys_in = isect_ids.contiguous()
    vals_in = gaussian_ids.to(torch.int32).contiguous()
    ws = workspace(lib.query("hx_sort_pairs_workspace_bytes", n, 8), dev)
    with torch.cuda.device(dev):
        lib.call("hx_sort_pairs_u64", ptr(keys_in), ptr(vals_in), ptr(keys_out), ptr(vals_out), n,
                 begin, 32 + tile_bits, ptr(ws), ws.numel(), stream(dev))
    return keys_out, vals_out


def bin_and_sort_gaussians(
    num_points: int,
    num_intersects: int,
    xys: Tensor,
    radii: Tensor,
    cum_tiles_hit: Tensor,
    tile_bounds: Tuple[int, int, int],
) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Unsorted and sorted (key, Gaussian id) lists plus tile bins, as in the
    reference (gsplat/utils.py:118-162)."""
    isect_ids, gaussian_ids = map_gaussian_to_intersects(
        num_points, num_intersects, xys, radii, cum_tiles_hit, tile_bounds
    )
    num_tiles = tile_bounds[0] * tile_bounds[1]
    isect_ids_sorted, gaussian_ids_sorted = sort_intersections(isect_ids, gaussian_ids, num_tiles)
    tile_bins = get_tile_bin_edges(num_intersects, num_tiles, isect_ids_sorted)
    return isect_ids, gaussian_ids, isect_ids_sorted, gaussian_ids_sorted, tile_bins


def bin_gaussians_fused(
    num_points: int,
    num_intersects: int,
    xys: Tensor,
    radii: Tensor,
    cum_tiles_hit: Tensor,
    tile_bounds: Tuple[int, int, int],
    tile_rows: Tuple[int, int] | None = None,
    return_keys: bool = False,
):
    """Sorted Gaussian ids and tile bins in one pass of fused kernels
    (32-bit tile keys, ceil(log2(tiles)) sorted bits).  Same result as
    bin_and_sort_gaussians' sorted outputs.  `tile_rows` = [begin, end)
    restricts binning to a horizontal stripe of tile rows."""
    dev = xys.device
    tx, ty = int(tile_bounds[0]), int(tile_bounds[1])
    rb, re_ = (0, ty) if tile_rows is None else (int(tile_rows[0]), int(tile_rows[1]))
    ni = int(num_intersects)
    ids_sorted = torch.empty((ni,), dtype=torch.int32, device=dev)
    tile_bins = torch.empty((tx * ty, 2), dtype=torch.int32, device=dev)
    keys = torch.empty((ni,), dtype=torch.int64, device=dev) if return_keys else None
    ws = workspace(lib.query("hx_bin_gaussians_2d_workspace_bytes", ni, tx * ty), dev)
    with torch.cuda.device(dev):
        lib.call("hx_bin_gaussians_2d", int(num_points), ni, ptr(xys), ptr(radii),
                 ptr(cum_tiles_hit), tx, ty, rb, re_, ptr(ids_sorted), ptr(tile_bins), ptr(keys),
                 ptr(ws), ws.numel(), stream(dev))
    if return_keys:
        return ids_sorted, tile_bins, keys
    return ids_sorted, tile_bins


def count_tiles_in_rows(xys: Tensor, radii: Tensor, tile_bounds, tile_rows) -> Tensor:
    """Per-Gaussian number of tiles inside tile rows [begin, end)."""
    dev = xys.device
    n = xys.size(0)
    counts = torch.empty((n,), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        lib.call("hx_count_tiles_2d", n, ptr(xys), ptr(radii), int(tile_bounds[0]),
                 int(tile_bounds[1]), int(tile_rows[0]), int(tile_rows[1]), ptr(counts),
                 stream(dev))
    return counts
