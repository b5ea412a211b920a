"""CPU restatement of the 2D image-hexel path — TEST INFRASTRUCTURE (see oracle/__init__.py).

  hexagon SDF + edge id     gsplat/cuda/csrc/hexels_forward.cu:22-47
  alpha (scale/rot, affine) hexels_forward.cu:49-140
  top-K forward             hexels_forward.cu:169-859 (cached-minimum insertion,
                            empty-tile fast path, colour gradient, emission)
  backward                  gsplat/cuda/csrc/hexels_backward.cu:11-1387

Vectorised over pixels with float32 torch ops (float64 for finite-difference
checks via oracle.raster2d.set_precision).  exp results are flushed to zero
below FLT_MIN like the reference's fast-math build.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import raster2d as r2

TOP_K = 10
EPS = 1e-4
HA = np.float32(0.5) * np.float32(1.7320508)  # sqrt(3)/2 as the reference's float constant
HB = 0.5


def _f():
    return r2.f32


@dataclass
class HexParams:
    xys: torch.Tensor                     # (N,2) pixel centres
    colors: torch.Tensor                  # (N,C)
    scales: Optional[torch.Tensor] = None     # (N,2)
    rotation: Optional[torch.Tensor] = None   # (N,1)
    affines: Optional[torch.Tensor] = None    # (N,2,2) row-vector
    color_grads: Optional[torch.Tensor] = None  # (N,2,C)
    color_grad_scale: float = 0.0
    aa: float = 0.0
    softnesses: Optional[torch.Tensor] = None   # (N,) or (N,3)
    softness: float = 1.0
    sharpness: Optional[torch.Tensor] = None    # (N,) or (N,1)
    emission: Optional[torch.Tensor] = None     # (N,C)

    def soft3(self):
        n = self.xys.shape[0]
        f = _f()
        if self.softnesses is None or self.softnesses.numel() == 0:
            return torch.full((n, 3), self.softness, dtype=f)
        s = self.softnesses.to(f)
        if s.ndim == 1:
            return s[:, None].expand(n, 3)
        return s

    def sharp(self):
        n = self.xys.shape[0]
        if self.sharpness is None or self.sharpness.numel() == 0:
            return torch.zeros(n, dtype=_f())
        return self.sharpness.reshape(-1).to(_f())


def _local(p: HexParams, g, dx, dy):
    """(u_rot, v_rot, u_base, v_base, s_u, s_v, u, v) for primitives g at offsets."""
    f = _f()
    if p.affines is not None:
        a = p.affines.to(f).reshape(-1, 4)[g]
        u_base = dx * a[..., 0] + dy * a[..., 2]
        v_base = dx * a[..., 1] + dy * a[..., 3]
        u_rot = v_rot = torch.zeros_like(dx)
        if p.aa > 0:
            su = torch.rsqrt(1.0 + p.aa * (a[..., 0] * a[..., 0] + a[..., 2] * a[..., 2]))
            sv = torch.rsqrt(1.0 + p.aa * (a[..., 1] * a[..., 1] + a[..., 3] * a[..., 3]))
        else:
            su = sv = torch.ones_like(dx)
        extra = a
    else:
        rot = p.rotation.reshape(-1).to(f)[g]
        s_t, c_t = torch.sin(rot), torch.cos(rot)
        sc = p.scales.to(f)[g]
        sx = sc[..., 0] + 1e-8
        sy = sc[..., 1] + 1e-8
        u_rot = dx * c_t + dy * s_t
        v_rot = -dx * s_t + dy * c_t
        u_base = u_rot / sx
        v_base = v_rot / sy
        if p.aa > 0:
            su = torch.rsqrt(1.0 + p.aa * (1.0 / (sx * sx)))
            sv = torch.rsqrt(1.0 + p.aa * (1.0 / (sy * sy)))
        else:
            su = sv = torch.ones_like(dx)
        extra = (c_t, s_t, sx, sy)
    return u_rot, v_rot, u_base, v_base, su, sv, u_base * su, v_base * sv, extra


def hex_sdf(u, v):
    """hexels_forward.cu:22-47 -> (dist, edge id)."""
    d0 = v.abs()
    t1 = float(HA) * u + HB * v
    t2 = float(HA) * u - HB * v
    d1, d2 = t1.abs(), t2.abs()
    m = d1
    edge = torch.ones_like(u, dtype=torch.int64)
    take2 = d2 >= m
    m = torch.where(take2, d2, m)
    edge = torch.where(take2, 2, edge)
    take0 = d0 > m
    dist = torch.where(take0, d0, m) - 1.0
    edge = torch.where(take0, 0, edge)
    return dist, edge, t1, t2


def _alpha(p: HexParams, g, dx, dy):
    l = _local(p, g, dx, dy)
    u, v = l[6], l[7]
    dist, edge, _, _ = hex_sdf(u, v)
    soft = p.soft3()[g]
    se = torch.gather(soft, -1, edge[..., None])[..., 0]
    sig = 1.0 / (1.0 + r2._fexp(dist * se))
    sh = p.sharp()[g]
    peak = torch.where(sh > 0, r2._fexp(-sh * (u * u + v * v)), torch.zeros_like(u))
    alpha = torch.where(sh > 0, sig * peak, sig)
    return alpha, peak, l, dist, edge, se, sig


def _colors_at(p: HexParams, g, dx, dy):
    f = _f()
    base = p.colors.to(f)[g]
    if p.color_grads is None:
        return base
    cg = p.color_grads.to(f)[g]  # (...,2,C)
    return base + p.color_grad_scale * (dx[..., None] * cg[..., 0, :] + dy[..., None] * cg[..., 1, :])


def forward(p: HexParams, ids_sorted, tile_bins, img_h, img_w, tile_ids=None):
    """hexels_forward.cu:169-859 -> out_img, pixel_topk, weights_sum, entropy."""
    f = _f()
    tiles_x = (img_w + 15) // 16
    tiles_y = (img_h + 15) // 16
    bins = np.asarray(tile_bins)
    tl = r2._Tiles(r2.all_tiles((tiles_x, tiles_y)) if tile_ids is None else tile_ids, tiles_x,
                   img_h, img_w, bins)
    npix = tl.i.size
    C = p.colors.shape[1]
    ids = torch.full((npix, TOP_K), -1, dtype=torch.int64)
    vals = torch.zeros((npix, TOP_K), dtype=f)
    peaks = torch.zeros((npix, TOP_K), dtype=f)
    rows = torch.arange(npix)
    maxlen = int(tl.count.max()) if tl.count.size else 0
    pt = torch.from_numpy(tl.pix_tile)
    start = torch.from_numpy(tl.start)[pt]
    count = torch.from_numpy(tl.count)[pt]
    inside = torch.from_numpy(tl.inside)
    ids_sorted = torch.as_tensor(ids_sorted).to(torch.int64)
    xys = p.xys.to(f)
    for jj in range(maxlen):
        has = (jj < count) & inside
        pos = torch.where(has, start + jj, torch.zeros_like(start))
        g = torch.where(has, ids_sorted[pos], torch.zeros_like(pos))
        dx = xys[g, 0] - tl.px.to(f)
        dy = xys[g, 1] - tl.py.to(f)
        alpha, peak = _alpha(p, g, dx, dy)[:2]
        # insertion rule (first empty slot, else first minimum; strictly greater)
        empty = ids < 0
        has_empty = empty.any(1)
        first_empty = torch.argmax(empty.to(torch.int8), dim=1)
        masked = torch.where(empty, torch.full_like(vals, float("inf")), vals)
        first_min = torch.argmin(masked, dim=1)
        slot = torch.where(has_empty, first_empty, first_min)
        min_val = torch.where(has_empty, torch.full_like(alpha, -1.0), vals[rows, slot])
        ins = has & (alpha > min_val)
        r = rows[ins]
        ids[r, slot[ins]] = g[ins]
        vals[r, slot[ins]] = alpha[ins]
        peaks[r, slot[ins]] = peak[ins]
    valid = ids >= 0
    sum_val = torch.zeros(npix, dtype=f)
    for k in range(TOP_K):
        sum_val = sum_val + torch.where(valid[:, k], vals[:, k], 0.0)
    denom = (sum_val.double() + EPS).to(f)
    out = torch.zeros((npix, C), dtype=f)
    gk = ids.clamp(min=0)
    dxk = xys[gk, 0] - tl.px.to(f)[:, None]
    dyk = xys[gk, 1] - tl.py.to(f)[:, None]
    colk = _colors_at(p, gk, dxk, dyk)  # (P,K,C)
    for k in range(TOP_K):
        vis = vals[:, k] / denom
        out = out + torch.where(valid[:, k, None], colk[:, k] * vis[:, None], 0.0)
    if p.emission is not None and p.emission.numel() > 0:
        em = p.emission.to(f)[gk]
        for k in range(TOP_K):
            out = out + torch.where(valid[:, k, None], em[:, k] * peaks[:, k, None], 0.0)
    ent = torch.zeros(npix, dtype=f)
    for k in range(TOP_K):
        pk = vals[:, k] / denom
        ent = ent + torch.where(valid[:, k], -pk * torch.log(pk + 1e-7), 0.0)
    # empty tiles: zeros, -1, EPS, 0
    empty_tile = (count == 0)
    denom = torch.where(empty_tile, torch.tensor(float(np.float32(EPS)), dtype=f), denom)
    out_img = r2._scatter((img_h, img_w, C), tl, out)
    topk = torch.full((img_h, img_w, TOP_K), -1, dtype=torch.int32)
    topk[torch.from_numpy(tl.i[tl.inside]), torch.from_numpy(tl.j[tl.inside])] = \
        ids[inside].to(torch.int32)
    return out_img, topk, r2._scatter((img_h, img_w), tl, denom), r2._scatter((img_h, img_w), tl, ent)


def _sign(x):
    return torch.where(x > 0, 1.0, torch.where(x < 0, -1.0, 0.0)).to(x.dtype)


def backward(p: HexParams, v_output, v_weights_sum, v_entropy, pixel_topk, img_h, img_w):
    """hexels_backward.cu:233-1387.  Returns a dict of float64-accumulated
    gradients cast to the working precision."""
    f = _f()
    n, C = p.xys.shape[0], p.colors.shape[1]
    topk = pixel_topk.reshape(-1, TOP_K).to(torch.int64)
    P = topk.shape[0]
    ii, jj = torch.meshgrid(torch.arange(img_h), torch.arange(img_w), indexing="ij")
    px = jj.reshape(-1).to(f)[:, None]
    py = ii.reshape(-1).to(f)[:, None]
    vout = v_output.reshape(P, C).to(f)
    active = topk[:, 0] >= 0
    valid = (topk >= 0) & active[:, None]
    g = topk.clamp(min=0)
    xys = p.xys.to(f)
    dx = xys[g, 0] - px
    dy = xys[g, 1] - py
    alpha, peak, l, dist, edge, se, sig = _alpha(p, g, dx, dy)
    u_rot, v_rot, u_base, v_base, su, sv, u, v, extra = l
    alpha = torch.where(valid, alpha, 0.0)
    denom = torch.full((P,), float(np.float32(EPS)), dtype=f)
    for k in range(TOP_K):
        denom = denom + torch.where(valid[:, k], alpha[:, k], 0.0)
    norm_d = alpha / denom[:, None]
    colk = _colors_at(p, g, dx, dy)  # (P,K,C)
    v_norm_d = torch.zeros((P, TOP_K), dtype=f)
    for c in range(C):
        v_norm_d = v_norm_d + colk[..., c] * vout[:, None, c]
    grads = {}
    acc = {}

    def add(name, idx, vals, shape):
        if name not in acc:
            acc[name] = torch.zeros(shape, dtype=torch.float64)
        m = valid.reshape(-1)
        src = vals.reshape((m.numel(),) + tuple(shape[1:]))[m]
        acc[name].index_add_(0, idx.reshape(-1)[m], src.double())

    add("v_colors", g, norm_d[..., None] * vout[:, None, :], (n, C))
    has_em = p.emission is not None and p.emission.numel() > 0
    v_peak_emit = torch.zeros((P, TOP_K), dtype=f)
    sh = p.sharp()[g]
    if has_em:
        em = p.emission.to(f)[g]
        pe = torch.where(sh > 0, peak, 0.0)
        add("v_emission", g, torch.where((pe > 0)[..., None], pe[..., None] * vout[:, None, :],
                                         0.0), (n, C))
        ve = torch.zeros((P, TOP_K), dtype=f)
        for c in range(C):
            ve = ve + em[..., c] * vout[:, None, c]
        v_peak_emit = torch.where(pe > 0, ve, 0.0)
    v_xy_color = None
    if p.color_grads is not None:
        cgs = p.color_grad_scale
        cg = p.color_grads.to(f)[g]
        add("v_color_grads", g, torch.stack([
            norm_d[..., None] * vout[:, None, :] * cgs * dx[..., None],
            norm_d[..., None] * vout[:, None, :] * cgs * dy[..., None]], -2), (n, 2, C))
        vdx = torch.zeros((P, TOP_K), dtype=f)
        vdy = torch.zeros((P, TOP_K), dtype=f)
        for c in range(C):
            vdx = vdx + norm_d * vout[:, None, c] * cgs * cg[..., 0, c]
            vdy = vdy + norm_d * vout[:, None, c] * cgs * cg[..., 1, c]
        v_xy_color = torch.stack([vdx, vdy], -1)
    v_d = v_norm_d / denom[:, None]
    v_d_sum = torch.zeros(P, dtype=f)
    for k in range(TOP_K):
        v_d_sum = v_d_sum + torch.where(valid[:, k], -alpha[:, k] / (denom * denom) * v_norm_d[:, k],
                                        0.0)
    v_d = v_d + v_d_sum[:, None]
    if v_weights_sum is not None:
        v_d = v_d + torch.where(valid, v_weights_sum.reshape(P, 1).to(f), 0.0)
    if v_entropy is not None:
        pk = alpha / denom[:, None]
        dhdp = torch.where(valid, -(torch.log(pk + 1e-7) + 1.0), 0.0)
        avg = torch.zeros(P, dtype=f)
        for k in range(TOP_K):
            avg = avg + torch.where(valid[:, k], pk[:, k] * dhdp[:, k], 0.0)
        v_d = v_d + torch.where(valid, v_entropy.reshape(P, 1).to(f) *
                                ((dhdp - avg[:, None]) / denom[:, None]), 0.0)
    # SDF partials
    du = torch.where(edge == 0, 0.0, float(HA) * torch.where(
        edge == 1, _sign(float(HA) * u + HB * v), _sign(float(HA) * u - HB * v)))
    dv = torch.where(edge == 0, _sign(v), torch.where(
        edge == 1, HB * _sign(float(HA) * u + HB * v), -HB * _sign(float(HA) * u - HB * v)))
    v_sig = torch.where(sh > 0, v_d * peak, v_d)
    v_peak = v_d * sig + v_peak_emit
    v_r2 = v_peak * peak * (-sh)
    v_u_peak = torch.where(sh > 0, v_r2 * 2.0 * u, 0.0)
    v_v_peak = torch.where(sh > 0, v_r2 * 2.0 * v, 0.0)
    if p.sharpness is not None and p.sharpness.numel() > 0:
        add("v_sharpness", g, torch.where(sh > 0, v_peak * peak * (-(u * u + v * v)), 0.0), (n, 1))
    if p.softnesses is not None and p.softnesses.numel() > 0:
        v_soft = v_sig * (-dist) * sig * (1.0 - sig)
        if p.softnesses.ndim == 2:
            oh = torch.nn.functional.one_hot(edge, 3).to(f) * v_soft[..., None]
            add("v_softnesses", g, oh, (n, 3))
        else:
            add("v_softnesses", g, v_soft, (n,))
    v_dist = v_sig * (-se) * sig * (1.0 - sig)
    v_u = v_dist * du + v_u_peak
    v_v = v_dist * dv + v_v_peak
    v_u_base = v_u * su
    v_v_base = v_v * sv
    v_s_u = v_u * u_base
    v_s_v = v_v * v_base
    if p.affines is not None:
        a = extra
        v_dx = v_u_base * a[..., 0] + v_v_base * a[..., 1]
        v_dy = v_u_base * a[..., 2] + v_v_base * a[..., 3]
        va = torch.stack([dx * v_u_base, dx * v_v_base, dy * v_u_base, dy * v_v_base], -1)
        if p.aa > 0:
            su3, sv3 = su * su * su, sv * sv * sv
            va = va + torch.stack([v_s_u * (-p.aa * a[..., 0] * su3),
                                   v_s_v * (-p.aa * a[..., 1] * sv3),
                                   v_s_u * (-p.aa * a[..., 2] * su3),
                                   v_s_v * (-p.aa * a[..., 3] * sv3)], -1)
        add("v_affines", g, va, (n, 4))
    else:
        c_t, s_t, sx, sy = extra
        inv_sx, inv_sy = 1.0 / sx, 1.0 / sy
        v_u_rot = v_u_base * inv_sx
        v_v_rot = v_v_base * inv_sy
        v_sx = v_u_base * (-u_rot) * inv_sx * inv_sx
        v_sy = v_v_base * (-v_rot) * inv_sy * inv_sy
        if p.aa > 0:
            v_sx = v_sx + v_s_u * (p.aa * (su * su * su) * (inv_sx * inv_sx * inv_sx))
            v_sy = v_sy + v_s_v * (p.aa * (sv * sv * sv) * (inv_sy * inv_sy * inv_sy))
        v_dx = v_u_rot * c_t + v_v_rot * (-s_t)
        v_dy = v_u_rot * s_t + v_v_rot * c_t
        add("v_scale", g, torch.stack([v_sx, v_sy], -1), (n, 2))
        add("v_rot", g, v_u_rot * v_rot + v_v_rot * (-u_rot), (n, 1))
    vxy = torch.stack([v_dx, v_dy], -1)
    if v_xy_color is not None:
        vxy = vxy + v_xy_color
    add("v_xy", g, vxy, (n, 2))
    for k2, t in acc.items():
        grads[k2] = t.to(f)
    return grads
