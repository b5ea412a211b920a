"""gsplat — B200-native (sm_100a) drop-in for the ``gsplat`` import of
honeycomb-surfels/hexel-kernel.

Same public functions and signatures as the reference's gsplat/__init__.py;
every kernel behind them is hand-written CUDA for sm_100a in
``libhexel_b200.so`` (no CPU fallback).
"""

from typing import Any
import warnings

import torch

from .project_gaussians_2d_scale_rot import project_gaussians_2d_scale_rot
from .rasterize_sum import rasterize_gaussians_sum
from .rasterize_no_tiles import rasterize_gaussians_no_tiles, rasterize_gaussians_simple
from .utils import (
    map_gaussian_to_intersects,
    bin_and_sort_gaussians,
    compute_cumulative_intersects,
    compute_cov2d_bounds,
    get_tile_bin_edges,
)
from .rasterize_hexels3d import *  # noqa: F401,F403
from .rasterize_hexels3d import __all__ as _hexels3d_all

__all__ = [
    "project_gaussians_2d_scale_rot",
    "rasterize_gaussians_sum",
    "rasterize_gaussians_no_tiles",
    "rasterize_gaussians_simple",
    *_hexels3d_all,
    "bin_and_sort_gaussians",
    "compute_cumulative_intersects",
    "compute_cov2d_bounds",
    "get_tile_bin_edges",
    "map_gaussian_to_intersects",
    "ProjectGaussians2dScaleRot",
    "RasterizeGaussiansSum",
    "BinAndSortGaussians",
    "ComputeCumulativeIntersects",
    "ComputeCov2dBounds",
    "GetTileBinEdges",
    "MapGaussiansToIntersects",
]


def _deprecated(name: str, replacement: str, fn):
    """Autograd-Function shim kept for backwards compatibility
    (reference gsplat/__init__.py:61-160): warns, forwards, has no backward."""

    class _Shim(torch.autograd.Function):
        @staticmethod
        def forward(ctx, *args, **kwargs):
            warnings.warn(
                f"{name} is deprecated, use {replacement} instead", DeprecationWarning
            )
            return fn(*args, **kwargs)

        @staticmethod
        def backward(ctx: Any, *grad_outputs: Any) -> Any:
            raise NotImplementedError

    _Shim.__name__ = name
    _Shim.__qualname__ = name
    return _Shim


MapGaussiansToIntersects = _deprecated(
    "MapGaussiansToIntersects", "map_gaussian_to_intersects", map_gaussian_to_intersects)
ComputeCumulativeIntersects = _deprecated(
    "ComputeCumulativeIntersects", "compute_cumulative_intersects", compute_cumulative_intersects)
ComputeCov2dBounds = _deprecated("ComputeCov2dBounds", "compute_cov2d_bounds", compute_cov2d_bounds)
GetTileBinEdges = _deprecated("GetTileBinEdges", "get_tile_bin_edges", get_tile_bin_edges)
BinAndSortGaussians = _deprecated(
    "BinAndSortGaussians", "bin_and_sort_gaussians", bin_and_sort_gaussians)
ProjectGaussians2dScaleRot = _deprecated(
    "ProjectGaussians2dScaleRot", "project_gaussians_2d_scale_rot", project_gaussians_2d_scale_rot)
RasterizeGaussiansSum = _deprecated(
    "RasterizeGaussiansSum", "rasterize_gaussians", rasterize_gaussians_sum)
