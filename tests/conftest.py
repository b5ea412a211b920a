"""Test configuration: import paths, the `gpu` marker and shared helpers."""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hexel-kernel_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def assert_grad_parity(mine, ref, exact=None, name: str = ""):
    """Gradient parity against the reference kernels.

    Both sides sum per-pixel contributions with fp32 atomics in different
    orders, so entries that cancel to near zero carry absolute noise
    proportional to the magnitude of the summed terms.  Criterion, per entry:
        |mine - ref| <= 1e-4 * |ref| + 1e-5 * max|ref|
    and, when the float64 oracle `exact` is given, ours must be about as
    accurate as the reference.  Both sum float32 atomics in an unspecified
    order, so the single worst entry varies from run to run; the check is on
    the root-mean-square error, with a looser bound on the maximum:
        rms|mine - exact| <= 2 * rms|ref - exact| + 1e-7 * max|exact|,
        max|mine - exact| <= 4 * max|ref - exact| + 1e-6 * max|exact|.
    """
    import torch

    a = mine.detach().double().cpu().reshape(-1)
    b = ref.detach().double().cpu().reshape(-1)
    assert a.shape == b.shape, name
    scale = float(b.abs().max()) if b.numel() else 0.0
    bound = 1e-4 * b.abs() + 1e-5 * scale
    bad = (a - b).abs() > bound
    assert not bool(bad.any()), (
        f"{name}: {int(bad.sum())}/{b.numel()} entries differ; max |diff| "
        f"{float((a - b).abs().max()):.3e}, scale {scale:.3e}")
    if exact is not None and exact.numel():
        e = exact.detach().double().cpu().reshape(-1)
        dm, dr = (a - e).abs(), (b - e).abs()
        emax = float(e.abs().max())
        rms_m, rms_r = float(dm.pow(2).mean().sqrt()), float(dr.pow(2).mean().sqrt())
        max_m, max_r = float(dm.max()), float(dr.max())
        assert rms_m <= 2 * rms_r + 1e-7 * emax, (
            f"{name}: rms error vs float64 oracle {rms_m:.3e} exceeds the reference's "
            f"{rms_r:.3e}")
        assert max_m <= 4 * max_r + 1e-6 * emax, (
            f"{name}: max error vs float64 oracle {max_m:.3e} exceeds the reference's "
            f"{max_r:.3e}")


GRAD_RTOL, GRAD_ATOL = 1e-4, 1e-6


def grad_compare_at_size(mine, ref, ref_again, name: str = "", rtol: float = GRAD_RTOL,
                         atol: float = GRAD_ATOL, k_worst: int = 8):
    """Gradient comparison at the benchmark sizes against the reference kernels.

    The stated criterion is, per entry, |mine - ref| <= rtol |ref| or
    |mine - ref| <= atol (1e-4 relative, 1e-6 absolute near zero).  Both
    sides sum float32 atomics in an unspecified order, so at these sizes the
    reference does not meet that criterion against itself either:
    `ref_again` is a second run of the reference on the same inputs.  Returns
    the figures (no assertion): entries outside the stated criterion for ours
    against the reference (`n_out`) and for the reference against itself
    (`n_out_ref`), the largest differences, and the flat indices of the
    `k_worst` entries by how far they exceed the criterion (`worst`), which
    callers settle against the float64 oracle (assert_grad_at_size)."""
    import torch

    a = mine.detach().double().cpu().reshape(-1)
    b = ref.detach().double().cpu().reshape(-1)
    c = ref_again.detach().double().cpu().reshape(-1)
    assert a.shape == b.shape == c.shape, name
    st = {"name": name, "numel": b.numel()}
    if b.numel() == 0:
        return st
    bound = torch.maximum(rtol * b.abs(), torch.full_like(b, atol))
    d, dr = (a - b).abs(), (c - b).abs()
    excess = d / bound
    out = excess > 1
    st.update(max_abs=float(b.abs().max()), max_diff=float(d.max()),
              max_diff_ref=float(dr.max()), n_out=int(out.sum()),
              n_out_ref=int((dr > bound).sum()))
    k = min(k_worst, int(out.sum()))
    st["worst"] = torch.topk(excess, k).indices.tolist() if k else []
    st["_tensors"] = (a, b, c)
    return st


def assert_grad_at_size(st, exact=None, rtol: float = GRAD_RTOL, atol: float = GRAD_ATOL):
    """Pass/fail for grad_compare_at_size's figures.

    (1) Ours may leave the stated criterion at no more entries than three
        times the reference does against itself, plus 10 (the two runs of
        the reference share most of their summation order; ours and the
        reference share none of it).
    (2) The worst entries are settled against the float64 oracle: `exact`
        maps a flat index to (float64 value, float32 value of the oracle).
        Entries whose terms cancel heavily move far under float32 summation
        order alone, and single entries scatter, so the accuracy comparison
        is over the checked entries of the tensor together:
            rms(mine - exact) <= 2 rms(ref - exact) + rtol rms(exact) + atol
        (the reference's error taken as the larger of its two runs'), and no
        single entry beyond 8 times the larger of the reference's error and
        the float32 oracle's (a third summation order) + rtol |exact| + atol.
    The compared tensors are dropped from `st`, which then prints as JSON."""
    name = st["name"]
    if st["numel"] == 0:
        return st
    a, b, c = st.pop("_tensors")
    fails = []
    if st["n_out"] > 3 * st["n_out_ref"] + 10:
        fails.append(f"{name}: {st['n_out']}/{st['numel']} entries outside 1e-4 rel / 1e-6 abs "
                     f"against the reference, which leaves it at {st['n_out_ref']} against "
                     f"itself")
    if exact:
        rows = []
        em2 = eb2 = ex2 = 0.0
        for i, (e, o32) in exact.items():
            em = abs(float(a[i]) - e)
            er = max(abs(float(b[i]) - e), abs(float(c[i]) - e))
            eo = abs(o32 - e)
            rows.append({"i": i, "exact": e, "err_ours": em, "err_ref": er, "err_oracle32": eo})
            em2 += em * em
            eb2 += er * er
            ex2 += e * e
            if em > 8 * max(er, eo) + rtol * abs(e) + atol:
                fails.append(f"{name}[{i}]: ours {float(a[i]):.7g}, reference {float(b[i]):.7g} "
                             f"/ {float(c[i]):.7g}, float32 oracle {o32:.7g}, float64 oracle "
                             f"{e:.7g}")
        k = len(rows)
        rms_m, rms_b, rms_e = (em2 / k) ** 0.5, (eb2 / k) ** 0.5, (ex2 / k) ** 0.5
        st["float64_checked"] = rows
        st["rms_err_ours"], st["rms_err_ref"] = rms_m, rms_b
        if rms_m > 2 * rms_b + rtol * rms_e + atol:
            fails.append(f"{name}: rms error {rms_m:.3e} over {k} entries checked against the "
                         f"float64 oracle; the reference's is {rms_b:.3e}")
    assert not fails, "; ".join(fails)
    return st


def ref_module(name: str):
    """The reference's CUDA extension built from its sources into oracle/_ref
    (see oracle/build_ref.py), or None when it was not built."""
    import importlib.util

    d = os.path.join(ROOT, "oracle", "_ref")
    path = os.path.join(d, name + ".so")
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def assert_close_oracle(a, b, name: str = "", atol: float = 1e-5, frac: float = 0.999,
                        atol_max: float = 1e-4, rtol: float = 0.0):
    """Float outputs against the CPU oracle.  The oracle rounds each product
    separately where the CUDA build contracts into fused multiply-adds, and the
    ray-splat intersection (px*Tw - Tu, then a cross product) cancels
    catastrophically near a surfel's edge-on directions, so a few entries
    differ by more than fp32 noise elsewhere: at least `frac` of the entries
    must be within atol (+ rtol*|b|) and all within atol_max (+ rtol*|b|)."""
    import torch

    x = a.detach().double().cpu().reshape(-1)
    y = b.detach().double().cpu().reshape(-1)
    assert x.shape == y.shape, name
    err = (x - y).abs() - rtol * y.abs()
    ok = float((err <= atol).double().mean()) if y.numel() else 1.0
    worst = float(err.max()) if y.numel() else 0.0
    assert ok >= frac and worst <= atol_max, (
        f"{name}: {ok:.5f} of entries within {atol:g} (need {frac}), worst {worst:.3e} "
        f"(limit {atol_max:g})")
