"""CPU restatement of the 3D hexel surfel rasteriser — TEST INFRASTRUCTURE (see oracle/__init__.py).

Follows gsplat/cuda_hexels3d/csrc/hexels3d_forward.cu:
  constants                 19-41
  preprocess                57-551   (ray-splat transform 156-202, screen AABB 204-219,
                                      hexagon bounds with near-plane clipping 221-258,
                                      tile rectangles 80-91, per-surfel setup 372-551)
  binning                   553-604  ((tile << 32 | depth bits) keys, stable sort, ranges)
  forward compositing       610-1011 (colour, overdraw, owner and surface outputs)
  backward                  1749-2492 (reverse traversal), 2494-2664 (geometry VJPs)

The forward is restated expression by expression; every tile's 16x16 pixels
are processed together against the tile's sorted surfel list, and the
per-pixel sequential semantics (alpha threshold, early termination at
transmittance 1e-4, median index, distortion moments) are kept exactly.

The backward is the reverse-mode derivative of that restated forward, taken
per (pixel, surfel) pair with torch.autograd (float64 for finite-difference
checks), plus the reference's departures from the exact derivative, which
are restated explicitly:
  * a pair whose screen-space prefilter alpha wins (use_filter) contributes no
    view-direction, normal, depth or distortion-depth gradient
    (hexels3d_forward.cu:2219-2260,2287-2342,2355-2368); its median-depth
    gradient goes to T[8] (2343-2351);
  * the overdraw term of the surfel that terminates a pixel is part of the
    forward sum but has no gradient (the backward visits list indices below
    the pixel's last index only, 1983-1991);
  * means2d is a screen-space proxy, dL/dT[2] * depth * W/2 and
    dL/dT[5] * depth * H/2 (2608-2626), and its fourth column accumulates the
    per-pair norm of that proxy (2456-2461).
"""

from __future__ import annotations

from typing import Callable, Dict, Optional

import numpy as np
import torch

BLOCK = 16
NEAR = 0.2
FAR = 100.0
FILTER_SIZE = 0.707106
FILTER_INV_SQ = 2.0
HEX_RADIUS = 1.15470053838
LOG254 = 5.537334267
FLT_EPS = float(np.finfo(np.float32).eps)
FLT_MAX = float(np.finfo(np.float32).max)
T_MIN = 1e-4
ALPHA_MIN = 1.0 / 255.0

f32 = torch.float32


def set_precision(dtype: torch.dtype) -> None:
    """Working precision of the floating-point restatement (float32; float64
    for finite-difference checks)."""
    global f32
    f32 = dtype


# --------------------------------------------------------------------------
# geometry (hexels3d_forward.cu:101-202)
# --------------------------------------------------------------------------
def quat_to_rotmat(q: torch.Tensor) -> torch.Tensor:
    """(P,4) quaternions packed (w, x, y, z), normalised -> (P,3,3) rotation
    matrices R[:, row, col] (hexels3d_forward.cu:101-125)."""
    s = 1.0 / torch.sqrt((q * q).sum(-1))
    w, x, y, z = q[:, 0] * s, q[:, 1] * s, q[:, 2] * s, q[:, 3] * s
    c0 = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y + w * z), 2 * (x * z - w * y)], -1)
    c1 = torch.stack([2 * (x * y - w * z), 1 - 2 * (x * x + z * z), 2 * (y * z + w * x)], -1)
    c2 = torch.stack([2 * (x * z + w * y), 2 * (y * z - w * x), 1 - 2 * (x * x + y * y)], -1)
    return torch.stack([c0, c1, c2], -1)


def transmat(means3d, scales, rotations, projmatrix, W: int, H: int, mod: float = 1.0):
    """Ray-splat transform T = S2W^T . M_proj . N2P stored as the reference
    stores it (row c holds column c of T): (P,9) with Tu = [0:3], Tv = [3:6],
    Tw = [6:9] (hexels3d_forward.cu:156-202)."""
    P = means3d.shape[0]
    dt = means3d.dtype
    R = quat_to_rotmat(rotations)
    s2w = torch.zeros((P, 4, 3), dtype=dt)
    s2w[:, :3, 0] = R[:, :, 0] * (mod * scales[:, 0:1])
    s2w[:, :3, 1] = R[:, :, 1] * (mod * scales[:, 1:2])
    s2w[:, :3, 2] = means3d
    s2w[:, 3, 2] = 1.0
    pm = projmatrix.reshape(4, 4).to(dt)
    n2p = torch.zeros((4, 3), dtype=dt)
    n2p[0, 0] = W / 2.0
    n2p[3, 0] = (W - 1.0) / 2.0
    n2p[1, 1] = H / 2.0
    n2p[3, 1] = (H - 1.0) / 2.0
    n2p[3, 2] = 1.0
    T = s2w.transpose(1, 2) @ pm @ n2p
    return T.transpose(1, 2).reshape(P, 9)


def view_dirs_of(means3d, campos):
    d = means3d - campos.reshape(1, 3).to(means3d.dtype)
    return d / torch.sqrt((d * d).sum(-1, keepdim=True) + 1e-8)


def normals_of(rotations):
    return quat_to_rotmat(rotations)[:, :, 2]


def center_of(means3d, projmatrix, W: int, H: int):
    """Projected surfel centre in pixels (the prefilter centre,
    hexels3d_forward.cu:509-521)."""
    pm = projmatrix.reshape(-1).to(means3d.dtype)
    x, y, z = means3d[:, 0], means3d[:, 1], means3d[:, 2]
    cx = pm[0] * x + pm[4] * y + pm[8] * z + pm[12]
    cy = pm[1] * x + pm[5] * y + pm[9] * z + pm[13]
    cw = pm[3] * x + pm[7] * y + pm[11] * z + pm[15]
    inv_w = 1.0 / (cw + 1e-8)
    return torch.stack([(W / 2.0) * (cx * inv_w) + (W - 1.0) / 2.0,
                        (H / 2.0) * (cy * inv_w) + (H - 1.0) / 2.0], -1)


# --------------------------------------------------------------------------
# preprocess (hexels3d_forward.cu:372-551)
# --------------------------------------------------------------------------
def get_rect(p: np.ndarray, r: np.ndarray, grid):
    """Tile rectangle [min, max) of a box centred at p with half extents r
    (hexels3d_forward.cu:80-91); C truncating float -> int conversion."""
    gx, gy = grid

    def trunc(x):
        x = np.nan_to_num(x, nan=0.0, posinf=2.0**31 - 1, neginf=-(2.0**31))
        return np.clip(np.trunc(x), -(2.0**31), 2.0**31 - 1).astype(np.int64)

    p = p.astype(np.float32)
    r = r.astype(np.float32)
    fb = np.float32(BLOCK)
    x0 = np.minimum(gx, np.maximum(0, trunc((p[:, 0] - r[:, 0]) / fb)))
    y0 = np.minimum(gy, np.maximum(0, trunc((p[:, 1] - r[:, 1]) / fb)))
    x1 = np.minimum(gx, np.maximum(0, trunc((p[:, 0] + r[:, 0] + fb - np.float32(1)) / fb)))
    y1 = np.minimum(gy, np.maximum(0, trunc((p[:, 1] + r[:, 1] + fb - np.float32(1)) / fb)))
    return x0, y0, x1, y1


def _aabb(T: np.ndarray, cutoff: np.ndarray):
    """Screen-space centre and half extents at the cutoff
    (hexels3d_forward.cu:204-219)."""
    Tu, Tv, Tw = T[:, 0:3], T[:, 3:6], T[:, 6:9]
    c2 = (cutoff * cutoff).astype(np.float32)
    t = np.stack([c2, c2, -np.ones_like(c2)], -1)
    d = (t * (Tw * Tw)).sum(-1, dtype=np.float32)
    bounded = d < 0
    ok = d != 0
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        f = t / np.where(ok, d, np.float32(1))[:, None]
        px = (f * (Tu * Tw)).sum(-1, dtype=np.float32)
        py = (f * (Tv * Tw)).sum(-1, dtype=np.float32)
        h0x = px * px - (f * (Tu * Tu)).sum(-1, dtype=np.float32)
        h0y = py * py - (f * (Tv * Tv)).sum(-1, dtype=np.float32)
        ext = np.stack([np.sqrt(np.maximum(np.float32(1e-4), h0x)),
                        np.sqrt(np.maximum(np.float32(1e-4), h0y))], -1)
    return ok, np.stack([px, py], -1).astype(np.float32), ext.astype(np.float32), bounded


def _hex_bounds(T: np.ndarray, apothem: np.ndarray, W: int, H: int):
    """Bounds of the projected hexagon, clipped at the near plane
    (hexels3d_forward.cu:221-258)."""
    Tu, Tv, Tw = T[:, 0:3], T[:, 3:6], T[:, 6:9]
    ap = (apothem + np.float32(4e-5) * np.maximum(np.float32(1), np.abs(apothem))).astype(np.float32)
    ok = ap > 0
    r = np.float32(HEX_RADIUS) * ap
    h = np.float32(0.5) * r
    z0 = np.zeros_like(ap)
    vx = [r, h, -h, -r, -h, h]
    vy = [z0, ap, ap, z0, -ap, -ap]
    lox = np.full_like(ap, FLT_MAX)
    loy = np.full_like(ap, FLT_MAX)
    hix = np.full_like(ap, -FLT_MAX)
    hiy = np.full_like(ap, -FLT_MAX)
    one = np.ones_like(ap)
    near = np.float32(NEAR)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for i in range(6):
            j = (i + 1) % 6
            a = np.stack([vx[i], vy[i], one], -1)
            b = np.stack([vx[j], vy[j], one], -1)
            za = (a * Tw).sum(-1, dtype=np.float32)
            zb = (b * Tw).sum(-1, dtype=np.float32)
            inc = za >= near
            qx = (a * Tu).sum(-1, dtype=np.float32) / za
            qy = (a * Tv).sum(-1, dtype=np.float32) / za
            lox = np.where(inc, np.minimum(lox, qx), lox)
            loy = np.where(inc, np.minimum(loy, qy), loy)
            hix = np.where(inc, np.maximum(hix, qx), hix)
            hiy = np.where(inc, np.maximum(hiy, qy), hiy)
            cross = (za < near) != (zb < near)
            s = (near - za) / (zb - za)
            e = a + s[:, None] * (b - a)
            qx = (e * Tu).sum(-1, dtype=np.float32) / near
            qy = (e * Tv).sum(-1, dtype=np.float32) / near
            lox = np.where(cross, np.minimum(lox, qx), lox)
            loy = np.where(cross, np.minimum(loy, qy), loy)
            hix = np.where(cross, np.maximum(hix, qx), hix)
            hiy = np.where(cross, np.maximum(hiy, qy), hiy)
    ok &= ~((lox > W) | (loy > H) | (hix < -1) | (hiy < -1))
    lox = np.maximum(lox - 1, np.float32(-BLOCK))
    loy = np.maximum(loy - 1, np.float32(-BLOCK))
    hix = np.minimum(hix + 1, np.float32(W + BLOCK))
    hiy = np.minimum(hiy + 1, np.float32(H + BLOCK))
    center = np.stack([(lox + hix) * np.float32(0.5), (loy + hiy) * np.float32(0.5)], -1)
    with np.errstate(invalid="ignore"):
        rad = np.stack([np.ceil((hix - lox) * np.float32(0.5)) + 1,
                        np.ceil((hiy - loy) * np.float32(0.5)) + 1], -1)
    rad = np.where(ok[:, None], np.nan_to_num(rad), 0).astype(np.int64)
    return ok, center.astype(np.float32), rad


def preprocess(means3d, scales, rotations, opacities, viewmatrix, projmatrix, campos, W: int,
               H: int, softness: float = 10.0, softnesses=None, prefilter: bool = False,
               conservative: bool = False, scale_modifier: float = 1.0) -> Dict:
    """Per-surfel preprocess (hexels3d_forward.cu:372-551).  Returns numpy
    int arrays (radii, tile_radii, rect, tiles_touched) and torch float
    tensors (points_xy, depths, transMats, opacities, softnesses, view_dirs,
    normals, points_xy_center) in the reference's layouts."""
    P = means3d.shape[0]
    grid = ((W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK)
    with torch.no_grad():
        # float outputs in the working precision; bounds from their float32 values
        m = means3d.detach().to(f32)
        vm = viewmatrix.reshape(-1).float()
        mf = means3d.detach().float()
        pz = (vm[2] * mf[:, 0] + vm[6] * mf[:, 1] + vm[10] * mf[:, 2] + vm[14]).numpy()
        T_work = transmat(m, scales.detach().to(f32), rotations.detach().to(f32),
                          projmatrix.to(f32), W, H, scale_modifier)
        T = T_work.float().numpy()
        vd = view_dirs_of(m, campos.to(f32))
        nr = normals_of(rotations.detach().to(f32))
        center = center_of(m, projmatrix.to(f32), W, H)
    op = opacities.float().numpy()
    if softnesses is None or softnesses.numel() == 0:
        s3 = np.full((P, 3), softness, np.float32)
        stride = 1
    elif softnesses.dim() == 1:
        s3 = np.repeat(softnesses.float().numpy()[:, None], 3, 1)
        stride = 1
    else:
        s3 = softnesses.float().numpy().copy()
        stride = 3
    s3 = np.maximum(s3, np.float32(1e-4))
    smin = s3.min(1)
    smax = s3.max(1)
    cutoff = (np.float32(HEX_RADIUS) * (np.float32(1) + np.float32(LOG254) / smin)).astype(np.float32)
    old_bound, point, ext, bounded = _aabb(T, cutoff)
    rb = np.maximum(np.maximum(ext[:, 0], ext[:, 1]), cutoff * np.float32(FILTER_SIZE))
    if prefilter:
        rb = np.maximum(rb, np.float32(3 * FILTER_SIZE))
    with np.errstate(invalid="ignore"):
        radius = np.where(old_bound, np.nan_to_num(np.ceil(rb)), 0).astype(np.int64)
    x0, y0, x1, y1 = get_rect(point, np.stack([radius, radius], -1), grid)
    old_visible = old_bound & (x0 < x1) & (y0 < y1)
    corrected = conservative and not prefilter
    keep = (pz > NEAR) & (old_visible | corrected)
    # the reference writes radii here and does not clear it when a later test
    # (opacity, hexagon bounds, empty rectangle) culls the surfel
    radii = np.where(keep & old_visible, radius, 0)
    tr = np.stack([radius, radius], -1)
    if not prefilter:
        sel = bounded & (op <= 1.0)
        with np.errstate(invalid="ignore"):
            trx = np.minimum(radius, np.nan_to_num(np.ceil(np.maximum(ext[:, 0], cutoff * np.float32(FILTER_SIZE)))).astype(np.int64) + 1)
            try_ = np.minimum(radius, np.nan_to_num(np.ceil(np.maximum(ext[:, 1], cutoff * np.float32(FILTER_SIZE)))).astype(np.int64) + 1)
        tr = np.where(sel[:, None], np.stack([trx, try_], -1), tr)
        a0, b0, a1, b1 = get_rect(point, tr, grid)
        x0, y0, x1, y1 = (np.where(sel, a0, x0), np.where(sel, b0, y0), np.where(sel, a1, x1),
                          np.where(sel, b1, y1))
    if not prefilter:
        lx0, ly0, lx1, ly1 = x0, y0, x1, y1
        keep &= ~(op < np.float32(1.0 / 255.0))
        margin = (np.float32(LOG254) / smin).astype(np.float32)
        with np.errstate(invalid="ignore", divide="ignore"):
            lc = np.log((np.float32(255.0) * (np.float32(1) + np.float32(8) * np.float32(FLT_EPS)))
                        * op - np.float32(1)).astype(np.float32)
            alt = lc / np.where(lc < 0, smax, smin)
        margin = np.where(op > np.float32(1.0 / 255.0), alt, margin).astype(np.float32)
        ok, hc, hr = _hex_bounds(T, (np.float32(1) + margin).astype(np.float32), W, H)
        keep &= ok
        x0, y0, x1, y1 = get_rect(hc, hr, grid)
        point, tr = hc, hr
        if not corrected:
            x0, y0 = np.maximum(x0, lx0), np.maximum(y0, ly0)
            x1, y1 = np.minimum(x1, lx1), np.minimum(y1, ly1)
            keep &= (x0 < x1) & (y0 < y1)
            point = np.stack([(x0 + x1) * (BLOCK * 0.5), (y0 + y1) * (BLOCK * 0.5)], -1).astype(np.float32)
            tr = np.stack([(x1 - x0) * (BLOCK // 2), (y1 - y0) * (BLOCK // 2)], -1)
        else:
            radii = np.where(keep & ~old_visible, np.maximum(tr[:, 0], tr[:, 1]), radii)
    radii = radii.astype(np.int32)
    touched = np.where(keep, (y1 - y0) * (x1 - x0), 0).astype(np.int64)
    kf = torch.from_numpy(keep)
    zero = lambda t: torch.where(kf.view(-1, *([1] * (t.dim() - 1))), t, torch.zeros_like(t))  # noqa: E731
    soft_out = torch.from_numpy(s3) if stride == 3 else torch.from_numpy(s3[:, 0].copy())
    return {
        "keep": keep, "radii": radii, "tile_radii": np.where(keep[:, None], tr, 0).astype(np.int32),
        "rect": (np.where(keep, x0, 0), np.where(keep, y0, 0), np.where(keep, x1, 0),
                 np.where(keep, y1, 0)),
        "tiles_touched": touched,
        "points_xy": torch.from_numpy(np.where(keep[:, None], point, 0).astype(np.float32)),
        "depths": torch.from_numpy(np.where(keep, pz, 0).astype(np.float32)),
        "transMats": zero(T_work),
        "opacities": zero(opacities.detach().to(f32)),
        "softnesses": zero(soft_out), "softness_stride": stride,
        "view_dirs": vd, "normals": zero(nr), "points_xy_center": zero(center),
        "grid": grid, "W": W, "H": H,
    }


# --------------------------------------------------------------------------
# binning (hexels3d_forward.cu:553-604)
# --------------------------------------------------------------------------
def bin_surfels(pre: Dict, only_tiles: Optional[np.ndarray] = None):
    """Keys (tile << 32 | depth bits) for every tile of each kept surfel's
    rectangle, rows then columns, surfels in index order; stable sort; tile
    ranges.  With only_tiles, keys of other tiles are dropped (the sorted
    lists of the kept tiles are unchanged)."""
    gx, gy = pre["grid"]
    x0, y0, x1, y1 = pre["rect"]
    depth_bits = pre["depths"].numpy().view(np.uint32).astype(np.uint64)
    keep = pre["keep"] & ((x1 - x0) * (y1 - y0) > 0)
    want = None
    if only_tiles is not None:
        want = np.zeros(gx * gy, bool)
        want[only_tiles] = True
    sel = np.nonzero(keep)[0]
    wx = (x1 - x0)[sel]
    cnt = wx * (y1 - y0)[sel]
    ids = np.repeat(sel, cnt).astype(np.int32)
    first = np.repeat(np.cumsum(cnt) - cnt, cnt)
    local = np.arange(ids.size) - first
    wrep = np.repeat(wx, cnt)
    ty = y0[ids] + local // np.maximum(wrep, 1)
    tx = x0[ids] + local % np.maximum(wrep, 1)
    t = (ty * gx + tx).astype(np.uint64)
    if want is not None:
        m = want[t.astype(np.int64)]
        t, ids = t[m], ids[m]
    keys = (t << np.uint64(32)) | depth_bits[ids]
    order = np.argsort(keys, kind="stable")
    keys_s, ids_s = keys[order], ids[order]
    ranges = np.zeros((gx * gy, 2), np.int64)
    if keys_s.size:
        tiles = (keys_s >> np.uint64(32)).astype(np.int64)
        starts = np.searchsorted(tiles, np.arange(gx * gy), side="left")
        ends = np.searchsorted(tiles, np.arange(gx * gy), side="right")
        ranges[:, 0], ranges[:, 1] = starts, ends
        ranges[ends == starts] = 0
    return keys_s, ids_s, ranges


# --------------------------------------------------------------------------
# compositing of one tile (forward 610-1011; backward by autograd + the
# reference's departures listed in the module docstring)
# --------------------------------------------------------------------------
def _hex_sdf(u, v):
    a = float(np.float32(0.5) * np.float32(1.7320508))
    b = 0.5
    d0 = v.abs()
    t1 = a * u + b * v
    t2 = a * u - b * v
    d1, d2 = t1.abs(), t2.abs()
    pick2 = d2 >= d1
    m = torch.where(pick2, d2, d1)
    edge = torch.where(pick2, torch.full_like(u, 2, dtype=torch.long),
                       torch.full_like(u, 1, dtype=torch.long))
    e0 = d0 > m
    edge = torch.where(e0, torch.zeros_like(edge), edge)
    return torch.where(e0, d0, m) - 1.0, edge


def _bounded(u, v):
    dist, _ = _hex_sdf(u, v)
    rho = dist + 1.0
    inv = torch.where(rho > 1.0, 1.0 / torch.where(rho > 1.0, rho, torch.ones_like(rho)),
                      torch.ones_like(rho))
    return u * inv, v * inv


def _excl_cumprod(x):
    c = torch.cumprod(x, dim=1)
    return torch.cat([torch.ones_like(c[:, :1]), c[:, :-1]], 1), c


def _excl_cumsum(x):
    c = torch.cumsum(x, dim=1)
    return torch.cat([torch.zeros_like(c[:, :1]), c[:, :-1]], 1)


class _Opts:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def _tile(px, py, ids, S: Dict, o: _Opts, tile_loss: Optional[Callable], pix_index):
    """Composite one tile.  px, py: (n,) pixel coordinates; ids: (L,) sorted
    surfel ids.  S: per-surfel tensors.  Returns per-pixel outputs and, when
    tile_loss is given, per-surfel gradient contributions."""
    n, L = px.shape[0], ids.shape[0]
    dt = f32
    ids_t = torch.from_numpy(ids.astype(np.int64))
    leaves = {}

    def leaf(name, per_pair=False):
        t = S[name][ids_t].to(dt)
        if per_pair:
            t = t.unsqueeze(0).expand(n, *t.shape).clone()
        if tile_loss is not None:
            t = t.detach().requires_grad_(True)
            leaves[name] = t
        return t

    T = leaf("transMats", per_pair=True)  # (n, L, 9)
    op = leaf("opacities")
    soft = leaf("softnesses")
    col = leaf("colors")
    cg = leaf("color_grads") if o.color_model >= 1 else None
    cq = leaf("color_quads") if o.color_model >= 2 else None
    vg = leaf("view_grads") if o.use_view_grads else None
    vd = leaf("view_dirs") if (o.use_view_grads or o.view_model == 2 or o.surface) else None
    nr = leaf("normals") if (o.view_model == 2 or o.surface) else None
    ks = leaf("specular_ks") if o.view_model == 2 else None
    ls = leaf("specular_log_s") if o.view_model == 2 else None
    ctr = leaf("points_xy_center") if o.prefilter else None

    X = px.to(dt)[:, None]
    Y = py.to(dt)[:, None]
    Tu, Tv, Tw = T[..., 0:3], T[..., 3:6], T[..., 6:9]
    k = X[..., None] * Tw - Tu
    l = Y[..., None] * Tw - Tv
    p = torch.linalg.cross(k, l, dim=-1)
    valid = p[..., 2] != 0
    pz = torch.where(valid, p[..., 2], torch.ones_like(p[..., 2]))
    u = p[..., 0] / pz
    v = p[..., 1] / pz
    depth_sdf = (u * Tw[..., 0] + v * Tw[..., 1]) + Tw[..., 2]
    valid = valid & (depth_sdf >= NEAR)
    dist, edge = _hex_sdf(u, v)
    if o.stride == 3:
        s_e = torch.gather(soft.unsqueeze(0).expand(n, L, 3), 2, edge.unsqueeze(-1)).squeeze(-1)
    else:
        s_e = soft.unsqueeze(0).expand(n, L)
    boundary = torch.sigmoid(-(dist * s_e))  # 1 / (1 + exp(dist * softness))
    alpha_raw = op[None, :] * boundary
    alpha_sdf = torch.clamp(alpha_raw, max=0.99)
    alpha = alpha_sdf
    use_filter = torch.zeros((n, L), dtype=torch.bool)
    if o.prefilter:
        dx = X - ctr[None, :, 0]
        dy = Y - ctr[None, :, 1]
        G = torch.exp(-0.5 * FILTER_INV_SQ * (dx * dx + dy * dy))
        af = torch.clamp(op[None, :] * G, max=0.99)
        use_filter = af > alpha_sdf
        alpha = torch.where(use_filter, af, alpha_sdf)
    ok = valid & (alpha >= ALPHA_MIN)
    is_base = torch.from_numpy(ids < o.overdraw_base)[None, :].expand(n, L)
    uf = use_filter
    depth = torch.where(uf, Tw[..., 2], depth_sdf)

    with torch.no_grad():
        a_eff = torch.where(ok, alpha, torch.zeros_like(alpha))
        t_after = torch.cumprod(1.0 - a_eff, dim=1)
        term = ok & (t_after < T_MIN)
        stop = torch.where(term.any(1), term.to(torch.int8).argmax(1),
                           torch.full((n,), L, dtype=torch.long))
        j = torch.arange(L)[None, :]
        cmask = ok & (j < stop[:, None])
        last_index = torch.where(cmask, j + 1, torch.zeros_like(j)).max(1).values if L else \
            torch.zeros(n, dtype=torch.long)
        od_mask = ok & is_base & (alpha_sdf >= ALPHA_MIN) & (j <= stop[:, None])
        od_term = od_mask & (j == stop[:, None])
        if o.surface:
            sok = ok & is_base
            s_after = torch.cumprod(1.0 - torch.where(sok, alpha, torch.zeros_like(alpha)), 1)
            sterm = sok & (s_after < T_MIN)
            sstop = torch.where(sterm.any(1), sterm.to(torch.int8).argmax(1),
                                torch.full((n,), L, dtype=torch.long))
            smask = sok & (j < sstop[:, None])

    zeros = torch.zeros_like(alpha)
    a_c = torch.where(cmask, alpha, zeros)
    T_before, T_cum = _excl_cumprod(1.0 - a_c)
    T_final = T_cum[:, -1] if L else torch.ones(n, dtype=dt)
    w = a_c * T_before

    u_app = torch.where(uf, zeros, u)
    v_app = torch.where(uf, zeros, v)
    c = col[None, :, :].expand(n, L, 3)
    if cg is not None:
        c = c + u_app[..., None] * cg[None, :, 0, :] + v_app[..., None] * cg[None, :, 1, :]
    if cq is not None:
        ub, vb = (u_app, v_app) if o.color_model == 2 else _bounded(u_app, v_app)
        c = c + (ub * ub)[..., None] * cq[None, :, 0, :] + (ub * vb)[..., None] * cq[None, :, 1, :] \
            + (vb * vb)[..., None] * cq[None, :, 2, :]
    vd_pair = None
    if vd is not None:
        vd_pair = vd[None].expand(n, L, 3)
        vd_pair = torch.where(uf[..., None], vd_pair.detach(), vd_pair)
    if vg is not None:
        c = c + (vd_pair[..., None, :] * vg[None]).sum(-1)
    if o.view_model == 2:
        nl = nr[None].expand(n, L, 3)
        nl = torch.where(uf[..., None], nl.detach(), nl)
        cos_nv = torch.clamp(-(nl * vd_pair).sum(-1), min=0.0)
        s_exp = torch.exp(torch.clamp(ls, 0.0, 5.0))[None, :]
        safe = torch.where(cos_nv > 0, cos_nv, torch.ones_like(cos_nv))
        spec = torch.where(cos_nv > 0, safe ** s_exp, zeros)
        c = c + spec[..., None] * ks[None]
    out = {"color": (w[..., None] * c).sum(1) + T_final[:, None] * o.bg[None, :].to(dt),
           "final_T": T_final, "last_index": last_index}
    alpha_raw_od = torch.where(od_term, alpha_raw.detach(), alpha_raw)
    out["overdraw"] = torch.where(od_mask, alpha_raw_od, zeros).sum(1)
    out["overdraw_hits"] = od_mask.to(dt).sum(1)
    if o.contrib or o.owner:
        with torch.no_grad():
            wd = w.detach()
            out["contrib_pairs"] = wd
            if o.owner and L:
                best = wd.max(1)
                has = best.values > 0
                arg = best.indices
                rows = torch.arange(n)
                out["owner_id"] = torch.where(has, ids_t[arg], torch.full_like(arg, -1))
                out["owner_weight"] = torch.where(has, best.values, torch.zeros_like(best.values))
                out["owner_u"] = torch.where(has, u.detach()[rows, arg], torch.zeros(n, dtype=dt))
                out["owner_v"] = torch.where(has, v.detach()[rows, arg], torch.zeros(n, dtype=dt))
                out["owner_sdf"] = torch.where(has, dist.detach()[rows, arg], torch.zeros(n, dtype=dt))
                out["owner_depth"] = torch.where(has, depth.detach()[rows, arg],
                                                 torch.zeros(n, dtype=dt))
            elif o.owner:
                out.update(owner_id=torch.full((n,), -1, dtype=torch.long),
                           owner_weight=torch.zeros(n, dtype=dt), owner_u=torch.zeros(n, dtype=dt),
                           owner_v=torch.zeros(n, dtype=dt), owner_sdf=torch.zeros(n, dtype=dt),
                           owner_depth=torch.zeros(n, dtype=dt))
            out["total_alpha"] = 1.0 - T_final.detach()
    if o.surface:
        a_s = torch.where(smask, alpha, zeros)
        Ts_before, Ts_cum = _excl_cumprod(1.0 - a_s)
        Ts_final = Ts_cum[:, -1] if L else torch.ones(n, dtype=dt)
        ws = a_s * Ts_before
        depth_g = torch.where(uf, depth.detach(), depth)
        sign = torch.where((nr[None] * vd[None]).sum(-1).detach() > 0, -1.0, 1.0).to(dt)
        n_s = sign[..., None] * nr[None]
        n_s = torch.where(uf[..., None], n_s.detach(), n_s)
        out["depth"] = (ws * depth_g).sum(1)
        out["alpha"] = 1.0 - Ts_final
        out["normal"] = (ws[..., None] * n_s).sum(1)
        safe_d = torch.where(smask, depth_g, torch.ones_like(depth_g))
        mval = FAR / (FAR - NEAR) * (1.0 - NEAR / safe_d)
        M1 = _excl_cumsum(mval * ws)
        M2 = _excl_cumsum(mval * mval * ws)
        acc = 1.0 - Ts_before
        out["distortion"] = ((mval * mval * acc + M2 - 2.0 * mval * M1) * ws).sum(1)
        if o.median:
            with torch.no_grad():
                cand = smask & (Ts_before > 0.5)
                jj = torch.where(cand, j.expand(n, L), torch.full_like(j.expand(n, L), -1))
                med = jj.max(1).values if L else torch.full((n,), -1, dtype=torch.long)
            rows = torch.arange(n)
            picked = depth[rows, med.clamp(min=0)] if L else torch.zeros(n, dtype=dt)
            out["median"] = torch.where(med >= 0, picked, torch.zeros(n, dtype=dt))
    grads = None
    if tile_loss is not None:
        loss = tile_loss(out, pix_index)
        names = list(leaves.keys())
        gs = torch.autograd.grad(loss, [leaves[k] for k in names], allow_unused=True)
        grads = {}
        for name, g in zip(names, gs):
            if g is None:
                g = torch.zeros_like(leaves[name])
            if name == "transMats":
                gT = g
                grads["transMats"] = gT.sum(0)
                gx = gT[..., 2] * T.detach()[..., 8] * (0.5 * o.W)
                gy = gT[..., 5] * T.detach()[..., 8] * (0.5 * o.H)
                grads["abs_means2d"] = torch.sqrt(gx * gx + gy * gy).sum(0)
            else:
                grads[name] = g
        grads["ids"] = ids_t
    out = {k: (v.detach() if torch.is_tensor(v) else v) for k, v in out.items()}
    return out, grads


def render(pre: Dict, ranges: np.ndarray, point_list: np.ndarray, colors, background,
           color_grads=None, color_quads=None, view_grads=None, specular_ks=None,
           specular_log_s=None, color_model: int = 1, view_model: int = 1,
           use_view_grads: bool = True, surface: bool = False, median: bool = False,
           contrib: bool = False, owner: bool = False, overdraw_base: int = -1,
           prefilter: bool = False, tiles: Optional[np.ndarray] = None,
           upstream: Optional[Dict[str, torch.Tensor]] = None,
           loss_fn: Optional[Callable] = None) -> Dict:
    """Forward compositing over the given tiles (all by default) and, with
    `upstream` (full-image output gradients keyed color, overdraw, depth,
    alpha, normal, distortion, median) or `loss_fn(tile_outputs, pixel_ids)`,
    the render backward: gradients per surfel of the compositing inputs."""
    W, H = pre["W"], pre["H"]
    gx, gy = pre["grid"]
    P = colors.shape[0]
    dt = f32
    S = {"transMats": pre["transMats"].to(dt), "opacities": pre["opacities"].to(dt),
         "softnesses": pre["softnesses"].to(dt), "colors": colors.to(dt),
         "view_dirs": pre["view_dirs"].to(dt), "normals": pre["normals"].to(dt),
         "points_xy_center": pre["points_xy_center"].to(dt)}
    if color_grads is not None and color_grads.numel():
        S["color_grads"] = color_grads.to(dt).reshape(P, 2, 3)
    if color_quads is not None and color_quads.numel():
        S["color_quads"] = color_quads.to(dt).reshape(P, 3, 3)
    if view_grads is not None and view_grads.numel():
        S["view_grads"] = view_grads.to(dt).reshape(P, 3, 3)
    if specular_ks is not None and specular_ks.numel():
        S["specular_ks"] = specular_ks.to(dt).reshape(P, 3)
        S["specular_log_s"] = specular_log_s.to(dt).reshape(P)
    o = _Opts(color_model=color_model, view_model=view_model, use_view_grads=use_view_grads,
              surface=surface, median=median, contrib=contrib, owner=owner,
              overdraw_base=P if overdraw_base <= 0 or overdraw_base > P else overdraw_base,
              prefilter=prefilter, stride=pre["softness_stride"], bg=background, W=W, H=H)
    HW = H * W
    res = {"color": torch.zeros((3, HW), dtype=dt), "final_T": torch.ones(HW, dtype=dt),
           "last_index": torch.zeros(HW, dtype=torch.long),
           "overdraw": torch.zeros(HW, dtype=dt), "overdraw_hits": torch.zeros(HW, dtype=dt)}
    if surface:
        for name in ("depth", "alpha", "distortion") + (("median",) if median else ()):
            res[name] = torch.zeros(HW, dtype=dt)
        res["normal"] = torch.zeros((3, HW), dtype=dt)
    if contrib:
        res["contrib"] = torch.zeros(P, dtype=dt)
    if owner:
        res.update(owner_id=torch.full((HW,), -1, dtype=torch.long),
                   owner_weight=torch.zeros(HW, dtype=dt), owner_u=torch.zeros(HW, dtype=dt),
                   owner_v=torch.zeros(HW, dtype=dt), owner_sdf=torch.zeros(HW, dtype=dt),
                   owner_depth=torch.zeros(HW, dtype=dt), total_alpha=torch.zeros(HW, dtype=dt))
    want_grad = upstream is not None or loss_fn is not None
    G = {}
    if want_grad:
        for name in S:
            G[name] = torch.zeros_like(S[name])
        G["abs_means2d"] = torch.zeros(P, dtype=dt)
    if upstream is not None:
        up = {k: v.reshape(HW) if v.numel() == HW else v.reshape(-1, HW)
              for k, v in upstream.items() if v is not None and v.numel()}

        def loss_fn(out, pix):  # noqa: F811
            total = torch.zeros((), dtype=dt)
            for key, val in out.items():
                if key not in up or not torch.is_tensor(val) or not val.requires_grad:
                    continue
                g = up[key][..., pix].to(dt)
                total = total + (g.T * val if val.dim() == 2 else g * val).sum()
            return total

    tiles = np.arange(gx * gy) if tiles is None else np.asarray(tiles)
    for t in tiles:
        tx, ty = int(t % gx), int(t // gx)
        xs = torch.arange(tx * BLOCK, min((tx + 1) * BLOCK, W))
        ys = torch.arange(ty * BLOCK, min((ty + 1) * BLOCK, H))
        yy, xx = torch.meshgrid(ys, xs, indexing="ij")
        px, py = xx.reshape(-1), yy.reshape(-1)
        pix = py * W + px
        b, e = int(ranges[t, 0]), int(ranges[t, 1])
        ids = point_list[b:e]
        if ids.size == 0:
            # empty list: the background; every other output keeps its
            # initial value (transmittance 1, last index 0, zeros, owner -1)
            res["color"][:, pix] = background.to(dt)[:, None]
            continue
        out, gr = _tile(px, py, ids, S, o, loss_fn if want_grad else None, pix)
        res["color"][:, pix] = out["color"].T
        res["final_T"][pix] = out["final_T"]
        res["last_index"][pix] = out["last_index"]
        res["overdraw"][pix] = out["overdraw"]
        res["overdraw_hits"][pix] = out["overdraw_hits"]
        if surface:
            for name in ("depth", "alpha", "distortion") + (("median",) if median else ()):
                res[name][pix] = out[name]
            res["normal"][:, pix] = out["normal"].T
        if contrib and "contrib_pairs" in out:
            res["contrib"].index_add_(0, torch.from_numpy(ids.astype(np.int64)),
                                      out["contrib_pairs"].sum(0))
        if owner:
            for name in ("owner_id", "owner_weight", "owner_u", "owner_v", "owner_sdf",
                         "owner_depth", "total_alpha"):
                res[name][pix] = out[name]
        if gr is not None:
            idx = gr["ids"]
            for name, g in gr.items():
                if name == "ids":
                    continue
                G[name].index_add_(0, idx, g)
    res["grads"] = G if want_grad else None
    return res


# --------------------------------------------------------------------------
# geometry backward (hexels3d_forward.cu:2494-2664)
# --------------------------------------------------------------------------
def geometry_backward(means3d, scales, rotations, projmatrix, campos, W: int, H: int,
                      radii: np.ndarray, grad_T, grad_view_dirs, grad_normals=None,
                      grad_center=None, scale_modifier: float = 1.0):
    """VJP from the transform, view direction, normal (and prefilter centre)
    gradients to means3d, scales and rotations; surfels with radius 0 get no
    transform/view/normal gradient."""
    dt = f32
    m = means3d.detach().to(dt).requires_grad_(True)
    s = scales.detach().to(dt).requires_grad_(True)
    q = rotations.detach().to(dt).requires_grad_(True)
    live = torch.from_numpy(radii > 0).to(dt)
    T = transmat(m, s, q, projmatrix.to(dt), W, H, scale_modifier)
    total = (T * (grad_T.to(dt) * live[:, None])).sum()
    total = total + (view_dirs_of(m, campos.to(dt)) * (grad_view_dirs.to(dt) * live[:, None])).sum()
    if grad_normals is not None:
        total = total + (normals_of(q) * (grad_normals.to(dt) * live[:, None])).sum()
    if grad_center is not None:
        total = total + (center_of(m, projmatrix.to(dt), W, H) * grad_center.to(dt)).sum()
    gm, gs, gq = torch.autograd.grad(total, [m, s, q])
    return gm, gs, gq


def means2d_proxy(grad_T, transMats, radii: np.ndarray, W: int, H: int, abs_sum=None):
    """Screen-space gradient proxy of means2d (hexels3d_forward.cu:2608-2626)
    with the per-pair norm accumulator as a fourth column when given."""
    P = grad_T.shape[0]
    live = torch.from_numpy(radii > 0)
    out = torch.zeros((P, 4 if abs_sum is not None else 3), dtype=grad_T.dtype)
    depth = transMats[:, 8].to(grad_T.dtype)
    out[:, 0] = torch.where(live, grad_T[:, 2] * depth * (0.5 * W), out[:, 0])
    out[:, 1] = torch.where(live, grad_T[:, 5] * depth * (0.5 * H), out[:, 1])
    if abs_sum is not None:
        out[:, 3] = abs_sum.to(grad_T.dtype)
    return out


# --------------------------------------------------------------------------
# whole path
# --------------------------------------------------------------------------
def forward_backward(means3d, scales, rotations, opacities, colors, color_grads, view_grads,
                     background, cam, softness: float = 10.0, upstream=None, loss_fn=None,
                     surface: bool = False, median: bool = False, tiles=None,
                     softnesses=None, color_quads=None, specular_ks=None, specular_log_s=None,
                     color_model: int = 1, view_model: int = 1, use_view_grads: bool = True,
                     prefilter: bool = False, conservative: bool = False,
                     overdraw_base: int = -1, means2d_cols: int = 0, pre=None) -> Dict:
    """Preprocess -> binning -> compositing (-> backward when upstream
    gradients or a loss are given) for one camera (width, height,
    viewmatrix, projmatrix, campos attributes).  `pre` may carry a
    preprocess result computed elsewhere (e.g. by the CUDA path) to isolate
    the compositing comparison."""
    W, H = cam.width, cam.height
    if pre is None:
        pre = preprocess(means3d, scales, rotations, opacities, cam.viewmatrix, cam.projmatrix,
                         cam.campos, W, H, softness, softnesses, prefilter, conservative)
    _, point_list, ranges = bin_surfels(pre, tiles)
    r = render(pre, ranges, point_list, colors, background, color_grads, color_quads,
               view_grads, specular_ks, specular_log_s, color_model, view_model,
               use_view_grads, surface, median, overdraw_base=overdraw_base,
               prefilter=prefilter, tiles=tiles, upstream=upstream, loss_fn=loss_fn)
    r["pre"], r["ranges"], r["point_list"] = pre, ranges, point_list
    G = r.pop("grads")
    if G is None:
        return r
    need_n = surface or view_model == 2
    gm, gs, gq = geometry_backward(means3d, scales, rotations, cam.projmatrix, cam.campos, W, H,
                                   pre["radii"], G["transMats"], G["view_dirs"]
                                   if "view_dirs" in G else torch.zeros((means3d.shape[0], 3)),
                                   G["normals"] if need_n else None,
                                   G["points_xy_center"] if prefilter else None)
    r["grads"] = {
        "means3d": gm, "scales": gs, "rotations": gq, "colors": G["colors"],
        "color_grads": G.get("color_grads"), "color_quads": G.get("color_quads"),
        "view_grads": G.get("view_grads"), "specular_ks": G.get("specular_ks"),
        "specular_log_s": G.get("specular_log_s"), "opacities": G["opacities"],
        "softnesses": G["softnesses"] if softnesses is not None and softnesses.numel() else None,
        "transMats": G["transMats"], "view_dirs": G.get("view_dirs"),
        "normals": G.get("normals"), "points_xy_center": G.get("points_xy_center"),
        "abs_means2d": G["abs_means2d"],
    }
    if means2d_cols:
        r["grads"]["means2d"] = means2d_proxy(G["transMats"], pre["transMats"], pre["radii"], W, H,
                                              G["abs_means2d"] if means2d_cols == 4 else None)
    return r


def sample_fwd_bwd(w, cam, crop_tiles: int, target: torch.Tensor) -> float:
    """One fwd+bwd of the RGB fit loss mean((rgb - target)^2) over a
    crop_tiles x crop_tiles tile crop at the image centre (the CPU baseline
    sample): preprocess of all surfels, binning restricted to the crop,
    compositing, backward to the surfel parameters.  Returns the megapixels
    rendered."""
    W, H = cam.width, cam.height
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    x0 = max(0, gx // 2 - crop_tiles // 2)
    y0 = max(0, gy // 2 - crop_tiles // 2)
    xs = np.arange(x0, min(gx, x0 + crop_tiles))
    ys = np.arange(y0, min(gy, y0 + crop_tiles))
    tiles = (ys[:, None] * gx + xs[None, :]).reshape(-1)
    numel = 3 * H * W
    tgt = target.reshape(3, H * W)

    def loss_fn(out, pix):
        d = out["color"] - tgt[:, pix].T.to(f32)
        return (d * d).sum() / numel

    forward_backward(w.means3d, w.scales, w.rotations, w.opacities, w.colors, w.color_grads,
                     w.view_grads, w.background, cam, w.softness, loss_fn=loss_fn, tiles=tiles)
    npx = sum(min(BLOCK, H - int(t // gx) * BLOCK) * min(BLOCK, W - int(t % gx) * BLOCK)
              for t in tiles)
    return npx / 1e6


def sample_fwd_bwd_split(w, cam, crop_tiles: int, target: torch.Tensor) -> Dict:
    """The CPU baseline sample timed in its two parts, so that a full frame
    can be extrapolated honestly: the per-view fixed part (preprocess of all
    surfels, binning of the whole frame, geometry VJP of all surfels) is timed
    in full, and the per-pixel part (compositing and its backward) over a
    crop_tiles x crop_tiles tile crop at the image centre, with the RGB fit
    loss mean((rgb - target)^2).  Returns seconds of each part, the crop's
    and the frame's megapixels, and the frame time fixed + per-pixel x
    frame / crop."""
    import time

    W, H = cam.width, cam.height
    gx, gy = (W + BLOCK - 1) // BLOCK, (H + BLOCK - 1) // BLOCK
    x0 = max(0, gx // 2 - crop_tiles // 2)
    y0 = max(0, gy // 2 - crop_tiles // 2)
    xs = np.arange(x0, min(gx, x0 + crop_tiles))
    ys = np.arange(y0, min(gy, y0 + crop_tiles))
    tiles = (ys[:, None] * gx + xs[None, :]).reshape(-1)
    numel = 3 * H * W
    tgt = target.reshape(3, H * W)

    def loss_fn(out, pix):
        d = out["color"] - tgt[:, pix].T.to(f32)
        return (d * d).sum() / numel

    t0 = time.perf_counter()
    pre = preprocess(w.means3d, w.scales, w.rotations, w.opacities, cam.viewmatrix,
                     cam.projmatrix, cam.campos, W, H, w.softness)
    _, point_list, ranges = bin_surfels(pre, None)
    t1 = time.perf_counter()
    r = render(pre, ranges, point_list, w.colors, w.background, w.color_grads, None,
               w.view_grads, tiles=tiles, loss_fn=loss_fn)
    t2 = time.perf_counter()
    G = r["grads"]
    geometry_backward(w.means3d, w.scales, w.rotations, cam.projmatrix, cam.campos, W, H,
                      pre["radii"], G["transMats"], G["view_dirs"])
    t3 = time.perf_counter()
    crop_px = sum(min(BLOCK, H - int(t // gx) * BLOCK) * min(BLOCK, W - int(t % gx) * BLOCK)
                  for t in tiles)
    fixed, pixel = (t1 - t0) + (t3 - t2), t2 - t1
    return {"fixed_s": fixed, "pixel_s": pixel, "crop_mpix": crop_px / 1e6,
            "frame_mpix": W * H / 1e6, "frame_s": fixed + pixel * (W * H) / crop_px}
