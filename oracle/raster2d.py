"""CPU restatement of the Image-GS 2D path — TEST INFRASTRUCTURE (see oracle/__init__.py).

Covers, in reference order:
  projection          gsplat/cuda/csrc/foward2d.cu:9-59, helpers.cuh:11-68,265-289
  projection VJP      gsplat/cuda/csrc/backward2d.cu:53-100, helpers.cuh:71-82
  binning             gsplat/utils.py:96-162, forward.cu:13-71
  top-K forward       gsplat/cuda/csrc/forward.cu:172-320
  top-K backward      gsplat/cuda/csrc/backward.cu:159-316
  plain-sum fwd/bwd   forward.cu:76-170, backward.cu:23-157
  tile-less fwd/bwd   forward.cu:322-410, backward.cu:318-438

Pixels are vectorised: every tile's 16x16 pixels are processed together and
candidates are visited in list order, so the per-pixel sequential semantics
(top-K insertion, sticky validity) are kept exactly.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

TOP_K = 10
BLOCK = 16
EPS = 1e-4
EPS_NO_TILES = 1e-7

f32 = torch.float32


def set_precision(dtype: torch.dtype) -> None:
    """Switch the working precision (float64 is used by finite-difference
    checks of the backward passes; the restatement itself is float32)."""
    global f32
    f32 = dtype


# --------------------------------------------------------------------------
# projection (foward2d.cu:9-59)
# --------------------------------------------------------------------------
def _mat2_mul(a, b):
    """Column-major 2x2 product, entries summed over the inner index in order
    (the reference's GLM operator*).  a, b: (..., 2, 2) indexed [col][row]."""
    out = torch.empty_like(a)
    out[..., 0, 0] = a[..., 0, 0] * b[..., 0, 0] + a[..., 1, 0] * b[..., 0, 1]
    out[..., 0, 1] = a[..., 0, 1] * b[..., 0, 0] + a[..., 1, 1] * b[..., 0, 1]
    out[..., 1, 0] = a[..., 0, 0] * b[..., 1, 0] + a[..., 1, 0] * b[..., 1, 1]
    out[..., 1, 1] = a[..., 0, 1] * b[..., 1, 0] + a[..., 1, 1] * b[..., 1, 1]
    return out


def _t(a):
    return a.transpose(-1, -2)


def _rot2(rot):
    c, s = torch.cos(rot), torch.sin(rot)
    r = torch.zeros(rot.shape + (2, 2), dtype=f32)
    r[..., 0, 0] = c
    r[..., 1, 1] = c
    r[..., 0, 1] = -s
    r[..., 1, 0] = s
    return r


def _rot2_grad(rot):
    c, s = torch.cos(rot), torch.sin(rot)
    r = torch.zeros(rot.shape + (2, 2), dtype=f32)
    r[..., 0, 0] = -s
    r[..., 1, 1] = -s
    r[..., 0, 1] = -c
    r[..., 1, 0] = c
    return r


def _scale2(s):
    r = torch.zeros(s.shape[:-1] + (2, 2), dtype=f32)
    r[..., 0, 0] = s[..., 0]
    r[..., 1, 1] = s[..., 1]
    return r


def cov2d_bounds(cov):
    """helpers.cuh:45-68: conic, radius and ok flag of (N,3) covariances."""
    a, b_, c = cov[:, 0], cov[:, 1], cov[:, 2]
    det = a * c - b_ * b_
    ok = det != 0
    inv_det = 1.0 / torch.where(ok, det, torch.ones_like(det))
    conic = torch.stack([c * inv_det, -b_ * inv_det, a * inv_det], dim=1)
    b = 0.5 * (a + c)
    disc = torch.sqrt(torch.clamp(b * b - det, min=0.1))
    v1 = b + disc
    v2 = b - disc
    radius = torch.ceil(3.0 * torch.sqrt(torch.maximum(v1, v2)))
    conic = torch.where(ok[:, None], conic, torch.zeros_like(conic))
    radius = torch.where(ok, radius, torch.zeros_like(radius))
    return conic, radius, ok


def tile_rect(xys: np.ndarray, radius: np.ndarray, tiles_x: int, tiles_y: int):
    """helpers.cuh:11-43 in float32: [x0,x1) x [y0,y1) tile rectangle."""
    xys = np.asarray(xys, dtype=np.float32)
    r = np.asarray(radius, dtype=np.float32) / np.float32(BLOCK)
    cx = xys[:, 0] / np.float32(BLOCK)
    cy = xys[:, 1] / np.float32(BLOCK)

    def clamp(v, hi):
        with np.errstate(invalid="ignore", over="ignore"):
            t = np.trunc(v.astype(np.float64))
        t = np.nan_to_num(t, nan=0.0, posinf=2**31 - 1, neginf=-(2**31))
        t = np.clip(t, 0, hi)
        return t.astype(np.int64)

    one = np.float32(1)
    x0 = clamp((cx - r).astype(np.float32), tiles_x)
    x1 = clamp(((cx + r).astype(np.float32) + one).astype(np.float32), tiles_x)
    y0 = clamp((cy - r).astype(np.float32), tiles_y)
    y1 = clamp(((cy + r).astype(np.float32) + one).astype(np.float32), tiles_y)
    return x0, y0, x1, y1


def project_2d(means2d, scales2d, rotation, img_height, img_width, tile_bounds):
    """foward2d.cu:9-59 -> xys (N,2), radii (N,) int32, conics (N,3), num_tiles_hit (N,)."""
    means2d = means2d.to(f32)
    scales2d = scales2d.to(f32)
    rot = rotation.reshape(-1).to(f32)
    center = torch.stack([means2d[:, 0] * float(img_width), means2d[:, 1] * float(img_height)], 1)
    R = _rot2(rot)
    S = _scale2(scales2d)
    M = _mat2_mul(R, S)
    cov = _mat2_mul(M, _t(M))
    cov2d = torch.stack([cov[:, 0, 0], cov[:, 0, 1], cov[:, 1, 1]], 1)
    conic, radius, ok = cov2d_bounds(cov2d)
    xys = torch.where(ok[:, None], center, torch.zeros_like(center))
    radii = radius.to(torch.int32)
    x0, y0, x1, y1 = tile_rect(xys.numpy(), radius.numpy(), tile_bounds[0], tile_bounds[1])
    area = (x1 - x0) * (y1 - y0)
    num_tiles_hit = torch.from_numpy(np.where(ok.numpy() & (area > 0), area, 0).astype(np.int32))
    return xys, radii, conic, num_tiles_hit


def project_2d_backward(scales2d, rotation, img_height, img_width, radii, conics, v_xy, v_conic):
    """backward2d.cu:53-100 -> v_cov2d, v_mean2d, v_scale, v_rot (zeros where radii<=0)."""
    rot = rotation.reshape(-1).to(f32)
    X = torch.stack([conics[:, 0], conics[:, 1], conics[:, 1], conics[:, 2]], 1).view(-1, 2, 2)
    G = torch.stack([v_conic[:, 0], v_conic[:, 1], v_conic[:, 1], v_conic[:, 2]], 1).view(-1, 2, 2)
    vS = _mat2_mul(_mat2_mul(-X, G), X)
    g11 = vS[:, 0, 0]
    g12 = vS[:, 1, 0] + vS[:, 0, 1]
    g22 = vS[:, 1, 1]
    R, Rg, S = _rot2(rot), _rot2_grad(rot), _scale2(scales2d.to(f32))
    M = _mat2_mul(R, S)
    theta_g = _mat2_mul(_mat2_mul(Rg, S), _t(M)) + _mat2_mul(_mat2_mul(M, _t(S)), _t(Rg))
    z = torch.zeros_like(S)
    sxg = z.clone()
    sxg[:, 0, 0] = 2.0 * scales2d[:, 0]
    syg = z.clone()
    syg[:, 1, 1] = 2.0 * scales2d[:, 1]
    sig_x = _mat2_mul(_mat2_mul(R, sxg), _t(R))
    sig_y = _mat2_mul(_mat2_mul(R, syg), _t(R))
    v_scale = torch.stack([
        g11 * sig_x[:, 0, 0] + 2 * g12 * sig_x[:, 0, 1] + g22 * sig_x[:, 1, 1],
        g11 * sig_y[:, 0, 0] + 2 * g12 * sig_y[:, 0, 1] + g22 * sig_y[:, 1, 1],
    ], 1)
    v_rot = g11 * theta_g[:, 0, 0] + 2 * g12 * theta_g[:, 0, 1] + g22 * theta_g[:, 1, 1]
    v_mean = torch.stack([v_xy[:, 0] * float(img_width), v_xy[:, 1] * float(img_height)], 1)
    v_cov2d = torch.stack([g11, g12, g22], 1)
    keep = (radii > 0)
    k2 = keep[:, None]
    return (torch.where(k2, v_cov2d, 0.0), torch.where(k2, v_mean, 0.0),
            torch.where(k2, v_scale, 0.0), torch.where(keep, v_rot, 0.0)[:, None])


# --------------------------------------------------------------------------
# binning (utils.py:96-162, forward.cu:13-71)
# --------------------------------------------------------------------------
def map_intersects(xys, radii, num_tiles_hit, tile_bounds, tile_rows=None):
    """Unsorted (tile<<32 | 0) keys and Gaussian ids, Gaussian-major, tile rows
    then columns (forward.cu:13-44).  tile_rows restricts to a stripe."""
    xys = np.asarray(xys, dtype=np.float32)
    radii = np.asarray(radii).astype(np.int64)
    tx, ty = int(tile_bounds[0]), int(tile_bounds[1])
    x0, y0, x1, y1 = tile_rect(xys, radii.astype(np.float32), tx, ty)
    if tile_rows is not None:
        y0 = np.maximum(y0, tile_rows[0])
        y1 = np.minimum(y1, tile_rows[1])
    valid = (radii > 0) & (x1 > x0) & (y1 > y0)
    keys, ids = [], []
    for g in np.nonzero(valid)[0]:
        ys, xs = np.meshgrid(np.arange(y0[g], y1[g]), np.arange(x0[g], x1[g]), indexing="ij")
        tiles = (ys * tx + xs).reshape(-1).astype(np.int64)
        keys.append(tiles << 32)
        ids.append(np.full(tiles.shape, g, dtype=np.int32))
    if not keys:
        return np.zeros(0, np.int64), np.zeros(0, np.int32)
    return np.concatenate(keys), np.concatenate(ids)


def sort_and_bin(isect_ids: np.ndarray, gaussian_ids: np.ndarray, num_tiles: int):
    """Stable sort by key (the reference's torch.sort of distinct-by-tile keys
    keeps equal keys in input order), then tile ranges (forward.cu:49-71)."""
    order = np.argsort(isect_ids, kind="stable")
    keys_sorted = isect_ids[order]
    ids_sorted = gaussian_ids[order]
    bins = tile_bins_from_keys(keys_sorted, num_tiles)
    return keys_sorted, ids_sorted, bins


def tile_bins_from_keys(keys_sorted: np.ndarray, num_tiles: int) -> np.ndarray:
    bins = np.zeros((num_tiles, 2), dtype=np.int32)
    if keys_sorted.size == 0:
        return bins
    tiles = (keys_sorted >> 32).astype(np.int64)
    change = np.nonzero(np.diff(tiles))[0] + 1
    starts = np.concatenate([[0], change])
    ends = np.concatenate([change, [tiles.size]])
    bins[tiles[starts], 0] = starts
    bins[tiles[starts], 1] = ends
    return bins


# --------------------------------------------------------------------------
# compositing helpers
# --------------------------------------------------------------------------
class _Tiles:
    """Per-pixel bookkeeping for a set of 16x16 tiles."""

    def __init__(self, tile_ids: np.ndarray, tiles_x: int, img_h: int, img_w: int,
                 bins: np.ndarray):
        self.tile_ids = np.asarray(tile_ids, dtype=np.int64)
        r = np.arange(BLOCK)
        ty = (self.tile_ids // tiles_x)[:, None, None]
        tx = (self.tile_ids % tiles_x)[:, None, None]
        i = (ty * BLOCK + r[None, :, None]).repeat(BLOCK, 2)
        j = (tx * BLOCK + r[None, None, :]).repeat(BLOCK, 1)
        self.i = i.reshape(-1)
        self.j = j.reshape(-1)
        self.inside = (self.i < img_h) & (self.j < img_w)
        self.pix_tile = np.repeat(np.arange(len(self.tile_ids)), BLOCK * BLOCK)
        self.start = bins[self.tile_ids, 0].astype(np.int64)
        self.count = (bins[self.tile_ids, 1] - bins[self.tile_ids, 0]).astype(np.int64)
        self.px = torch.from_numpy(self.j.astype(np.float32))
        self.py = torch.from_numpy(self.i.astype(np.float32))


def _sigma(xy, conic, px, py):
    dx = xy[..., 0] - px
    dy = xy[..., 1] - py
    return (0.5 * (conic[..., 0] * dx * dx + conic[..., 2] * dy * dy) + conic[..., 1] * dx * dy,
            dx, dy)


FLT_MIN = 1.1754943508222875e-38


def _ftz(x):
    """Flush subnormal results to zero, as the reference's fast-math build
    (-ftz=true) does for every single-precision result."""
    if x.dtype != torch.float32:
        return x
    return torch.where(x.abs() < FLT_MIN, torch.zeros_like(x), x)


def _fexp(x):
    """exp() with the reference's flush-to-zero of subnormal results: weights
    of far-away primitives become exactly 0, which decides which of them fill
    empty top-K slots."""
    return _ftz(torch.exp(x))


def _bad(sigma):
    return (sigma < 0) | torch.isnan(sigma) | torch.isinf(sigma)


def _topk_select(cand_iter, npix):
    """Sequential top-K insertion (forward.cu:255-280), vectorised over pixels.

    cand_iter yields (g (P,) int64 with -1 = none, alpha (P,) float32)."""
    ids = torch.full((npix, TOP_K), -1, dtype=torch.int64)
    vals = torch.zeros((npix, TOP_K), dtype=f32)
    rows = torch.arange(npix)
    for g, alpha in cand_iter:
        empty = ids < 0
        has_empty = empty.any(1)
        first_empty = torch.argmax(empty.to(torch.int8), dim=1)
        masked = torch.where(empty, torch.full_like(vals, float("inf")), vals)
        first_min = torch.argmin(masked, dim=1)
        slot = torch.where(has_empty, first_empty, first_min)
        min_val = torch.where(has_empty, torch.full_like(alpha, -1.0), vals[rows, slot])
        ins = (g >= 0) & (alpha > min_val)
        r = rows[ins]
        ids[r, slot[ins]] = g[ins]
        vals[r, slot[ins]] = alpha[ins]
    return ids, vals


def _candidates(tl: _Tiles, ids_sorted: torch.Tensor, xys, conics):
    """Yields (g, sigma) for candidate j = 0, 1, ... of every pixel's tile."""
    maxlen = int(tl.count.max()) if tl.count.size else 0
    ids_sorted = ids_sorted.to(torch.int64)
    pt = torch.from_numpy(tl.pix_tile)
    start = torch.from_numpy(tl.start)[pt]
    count = torch.from_numpy(tl.count)[pt]
    inside = torch.from_numpy(tl.inside)
    for jj in range(maxlen):
        has = (jj < count) & inside
        pos = torch.where(has, start + jj, torch.zeros_like(start))
        g = torch.where(has, ids_sorted[pos], torch.full_like(pos, -1))
        gg = g.clamp(min=0)
        sigma, dx, dy = _sigma(xys[gg], conics[gg], tl.px, tl.py)
        yield g, sigma


def _scatter(img_shape, tl: _Tiles, values: torch.Tensor):
    out = torch.zeros(img_shape, dtype=values.dtype)
    m = torch.from_numpy(tl.inside)
    out[torch.from_numpy(tl.i[tl.inside]), torch.from_numpy(tl.j[tl.inside])] = values[m]
    return out


def all_tiles(tile_bounds) -> np.ndarray:
    return np.arange(int(tile_bounds[0]) * int(tile_bounds[1]))


def rasterize_topk_forward(xys, conics, colors, ids_sorted, tile_bins, img_h, img_w,
                           tile_ids: Optional[Sequence[int]] = None):
    """forward.cu:172-320 -> out_img (H,W,C), pixel_topk (H,W,10), weights_sum, entropy.

    tile_ids restricts the work to a subset of tiles (other pixels stay 0/-1)."""
    tiles_x = (img_w + BLOCK - 1) // BLOCK
    tiles_y = (img_h + BLOCK - 1) // BLOCK
    bins = np.asarray(tile_bins)
    tl = _Tiles(all_tiles((tiles_x, tiles_y)) if tile_ids is None else tile_ids, tiles_x, img_h,
                img_w, bins)
    xys = xys.to(f32)
    conics = conics.to(f32)
    colors = colors.to(f32)
    npix = tl.i.size

    def cands():
        for g, sigma in _candidates(tl, ids_sorted, xys, conics):
            ok = (g >= 0) & ~_bad(sigma)
            alpha = _fexp(-sigma)
            yield torch.where(ok, g, torch.full_like(g, -1)), alpha

    ids, vals = _topk_select(cands(), npix)
    valid = ids >= 0
    sum_val = torch.zeros(npix, dtype=f32)
    for k in range(TOP_K):
        sum_val = sum_val + torch.where(valid[:, k], vals[:, k], 0.0)
    denom = (sum_val.double() + EPS).to(f32)
    C = colors.shape[1]
    out = torch.zeros((npix, C), dtype=f32)
    for k in range(TOP_K):
        vis = vals[:, k] / denom
        col = colors[ids[:, k].clamp(min=0)]
        out = out + torch.where(valid[:, k, None], col * vis[:, None], 0.0)
    ent = torch.zeros(npix, dtype=f32)
    for k in range(TOP_K):
        p = vals[:, k] / denom
        ent = ent + torch.where(valid[:, k], -p * torch.log(p + 1e-7), 0.0)
    out_img = _scatter((img_h, img_w, C), tl, out)
    topk = torch.full((img_h, img_w, TOP_K), -1, dtype=torch.int32)
    topk[torch.from_numpy(tl.i[tl.inside]), torch.from_numpy(tl.j[tl.inside])] = \
        ids[torch.from_numpy(tl.inside)].to(torch.int32)
    ws = _scatter((img_h, img_w), tl, denom)
    en = _scatter((img_h, img_w), tl, ent)
    return out_img, topk, ws, en


def rasterize_topk_backward(xys, conics, colors, v_output, pixel_topk, img_h, img_w,
                            v_weights_sum=None, v_entropy=None, eps: float = EPS):
    """backward.cu:159-316 (eps=1e-4) and 318-438 (eps=1e-7, no aux terms).

    Returns v_xy (N,2), v_conic (N,3), v_colors (N,C) accumulated in float64
    and rounded to float32."""
    n, C = xys.shape[0], colors.shape[1]
    topk = pixel_topk.reshape(-1, TOP_K).to(torch.int64)
    P = topk.shape[0]
    ii, jj = torch.meshgrid(torch.arange(img_h), torch.arange(img_w), indexing="ij")
    px = jj.reshape(-1).to(f32)
    py = ii.reshape(-1).to(f32)
    vout = v_output.reshape(P, C).to(f32)
    valid = topk >= 0
    g = topk.clamp(min=0)
    xy = xys.to(f32)[g]        # (P,K,2)
    cn = conics.to(f32)[g]     # (P,K,3)
    sigma, dx, dy = _sigma(xy, cn, px[:, None], py[:, None])
    d = torch.where(valid, _fexp(-sigma), 0.0)
    denom = torch.full((P,), float(np.float32(eps)), dtype=f32)
    for k in range(TOP_K):
        denom = denom + torch.where(valid[:, k], d[:, k], 0.0)
    rgb = colors.to(f32)[g]    # (P,K,C)
    v_d = torch.zeros((P, TOP_K), dtype=f32)
    norm_d = d / denom[:, None]
    v_colors_pk = norm_d[:, :, None] * vout[:, None, :]
    v_norm_d = torch.zeros((P, TOP_K), dtype=f32)
    for c in range(C):
        v_norm_d = v_norm_d + rgb[:, :, c] * vout[:, None, c]
    for k in range(TOP_K):
        tmp = -d[:, k] / (denom * denom) * v_norm_d[:, k]
        add = torch.where(valid[:, k], tmp, 0.0)[:, None].expand(P, TOP_K).clone()
        add[:, k] = torch.where(valid[:, k], v_norm_d[:, k] / denom + tmp, 0.0)
        v_d = v_d + add
    if v_weights_sum is not None:
        v_d = v_d + torch.where(valid, v_weights_sum.reshape(P, 1).to(f32), 0.0)
    if v_entropy is not None:
        p = d / denom[:, None]
        dhdp = torch.where(valid, -(torch.log(p + 1e-7) + 1.0), 0.0)
        avg = torch.zeros(P, dtype=f32)
        for k in range(TOP_K):
            avg = avg + torch.where(valid[:, k], p[:, k] * dhdp[:, k], 0.0)
        dhdw = (dhdp - avg[:, None]) / denom[:, None]
        v_d = v_d + torch.where(valid, v_entropy.reshape(P, 1).to(f32) * dhdw, 0.0)
    v_sigma = v_d * -d
    v_conic_pk = torch.stack([0.5 * v_sigma * dx * dx, v_sigma * dx * dy,
                              0.5 * v_sigma * dy * dy], -1)
    v_xy_pk = torch.stack([v_sigma * (cn[..., 0] * dx + cn[..., 1] * dy),
                           v_sigma * (cn[..., 1] * dx + cn[..., 2] * dy)], -1)
    gv = g[valid]
    v_xy = torch.zeros((n, 2), dtype=torch.float64).index_add_(0, gv, v_xy_pk[valid].double())
    v_conic = torch.zeros((n, 3), dtype=torch.float64).index_add_(0, gv,
                                                                   v_conic_pk[valid].double())
    v_colors = torch.zeros((n, C), dtype=torch.float64).index_add_(0, gv,
                                                                    v_colors_pk[valid].double())
    return v_xy.to(f32), v_conic.to(f32), v_colors.to(f32)


def rasterize_sum_forward(xys, conics, colors, ids_sorted, tile_bins, img_h, img_w,
                          tile_ids=None):
    """forward.cu:76-170: plain sum of colour * exp(-sigma)."""
    tiles_x = (img_w + BLOCK - 1) // BLOCK
    tiles_y = (img_h + BLOCK - 1) // BLOCK
    tl = _Tiles(all_tiles((tiles_x, tiles_y)) if tile_ids is None else tile_ids, tiles_x, img_h,
                img_w, np.asarray(tile_bins))
    xys, conics, colors = xys.to(f32), conics.to(f32), colors.to(f32)
    out = torch.zeros((tl.i.size, colors.shape[1]), dtype=f32)
    for g, sigma in _candidates(tl, ids_sorted, xys, conics):
        ok = (g >= 0) & ~_bad(sigma)
        vis = _fexp(-sigma)
        out = out + torch.where(ok[:, None], colors[g.clamp(min=0)] * vis[:, None], 0.0)
    return _scatter((img_h, img_w, colors.shape[1]), tl, out)


def rasterize_sum_backward(xys, conics, colors, ids_sorted, tile_bins, v_output, img_h, img_w):
    """backward.cu:23-157 (validity is sticky per pixel, as in the reference)."""
    tiles_x = (img_w + BLOCK - 1) // BLOCK
    tiles_y = (img_h + BLOCK - 1) // BLOCK
    tl = _Tiles(all_tiles((tiles_x, tiles_y)), tiles_x, img_h, img_w, np.asarray(tile_bins))
    xys, conics, colors = xys.to(f32), conics.to(f32), colors.to(f32)
    n, C = xys.shape[0], colors.shape[1]
    inside = torch.from_numpy(tl.inside)
    pix = torch.from_numpy(np.minimum(tl.i * img_w + tl.j, img_w * img_h - 1))
    vout = v_output.reshape(-1, C).to(f32)[pix]
    valid = inside.clone()
    v_xy = torch.zeros((n, 2), dtype=torch.float64)
    v_conic = torch.zeros((n, 3), dtype=torch.float64)
    v_colors = torch.zeros((n, C), dtype=torch.float64)
    maxlen = int(tl.count.max()) if tl.count.size else 0
    pt = torch.from_numpy(tl.pix_tile)
    start = torch.from_numpy(tl.start)[pt]
    count = torch.from_numpy(tl.count)[pt]
    ids_sorted = ids_sorted.to(torch.int64)
    for jj in range(maxlen):
        has = jj < count
        pos = torch.where(has, start + jj, torch.zeros_like(start))
        g = torch.where(has, ids_sorted[pos], torch.zeros_like(pos))
        sigma, dx, dy = _sigma(xys[g], conics[g], tl.px, tl.py)
        d = _fexp(-sigma)
        valid = valid & ~(has & _bad(sigma))
        use = valid & has
        v_sigma = (colors[g] * vout).sum(1) * -d
        cn = conics[g]
        vc = torch.stack([0.5 * v_sigma * dx * dx, v_sigma * dx * dy, 0.5 * v_sigma * dy * dy], 1)
        vx = torch.stack([v_sigma * (cn[:, 0] * dx + cn[:, 1] * dy),
                          v_sigma * (cn[:, 1] * dx + cn[:, 2] * dy)], 1)
        vr = d[:, None] * vout
        gu = g[use]
        v_xy.index_add_(0, gu, vx[use].double())
        v_conic.index_add_(0, gu, vc[use].double())
        v_colors.index_add_(0, gu, vr[use].double())
    return v_xy.to(f32), v_conic.to(f32), v_colors.to(f32)


def rasterize_no_tiles_forward(xys, conics, colors, img_h, img_w):
    """forward.cu:322-410: top-K over all Gaussians, EPS 1e-7, double division."""
    xys, conics, colors = xys.to(f32), conics.to(f32), colors.to(f32)
    ii, jj = torch.meshgrid(torch.arange(img_h), torch.arange(img_w), indexing="ij")
    px = jj.reshape(-1).to(f32)
    py = ii.reshape(-1).to(f32)
    P = px.numel()

    def cands():
        for g in range(xys.shape[0]):
            sigma, _, _ = _sigma(xys[g], conics[g], px, py)
            ok = ~_bad(sigma)
            yield torch.where(ok, torch.full((P,), g), torch.full((P,), -1)), _fexp(-sigma)

    ids, vals = _topk_select(cands(), P)
    valid = ids >= 0
    sum_val = torch.zeros(P, dtype=f32)
    for k in range(TOP_K):
        sum_val = sum_val + torch.where(valid[:, k], vals[:, k], 0.0)
    out = torch.zeros((P, colors.shape[1]), dtype=f32)
    for k in range(TOP_K):
        vis = (vals[:, k].double() / (sum_val.double() + EPS_NO_TILES)).to(f32)
        out = out + torch.where(valid[:, k, None], colors[ids[:, k].clamp(min=0)] * vis[:, None],
                                0.0)
    return out.view(img_h, img_w, -1), ids.view(img_h, img_w, TOP_K).to(torch.int32)
