"""CPU checks of the C-ABI boundary: the library loads, exports every symbol
that include/hexel_b200.h declares, reports its ABI version and rejects bad
arguments with a status code and a message (no GPU work is launched)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hexel_b200.h")
LIB = os.path.join(ROOT, "hexel-kernel_b200", "gsplat", "libhexel_b200.so")


def declared():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return re.findall(r"HX_API\s+[\w\s\*]+?\s+\**(hx_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = declared()
    assert len(names) == len(set(names))
    assert "hx_nd_rasterize_forward_topk_norm" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_error_path():
    from gsplat._lib import lib, ABI_VERSION

    assert lib.dll.hx_abi_version() == ABI_VERSION
    with pytest.raises(RuntimeError, match="non-negative"):
        lib.call("hx_project_gaussians_2d_scale_rot_forward", -1, None, None, None, 4, 4, 1, 1,
                 None, None, None, None, None)
    with pytest.raises(RuntimeError, match="bit range"):
        lib.call("hx_sort_pairs_u64", None, None, None, None, 10, 0, 65, None, 0, None)
    with pytest.raises(RuntimeError, match="workspace"):
        lib.call("hx_sort_pairs_u32", 1, 1, 1, 1, 10, 0, 8, None, 0, None)


def test_python_surface_matches_reference_names():
    import gsplat
    import gsplat.cuda as C
    from gsplat import csrc

    two_d = """nd_rasterize_forward nd_rasterize_backward nd_rasterize_forward_topk_norm
    nd_rasterize_backward_topk_norm nd_rasterize_forward_topk_norm_stats
    nd_rasterize_backward_topk_norm_stats nd_rasterize_forward_no_tiles
    nd_rasterize_backward_no_tiles nd_rasterize_forward_simple nd_rasterize_backward_simple
    rasterize_forward rasterize_backward project_gaussians_2d_scale_rot_forward
    project_gaussians_2d_scale_rot_backward compute_cov2d_bounds map_gaussian_to_intersects
    get_tile_bin_edges""".split()
    for n in two_d:
        assert callable(getattr(csrc, n)), n
        assert callable(getattr(C, n)), n
    for n in ("project_gaussians_2d_scale_rot", "rasterize_gaussians_sum",
              "rasterize_gaussians_no_tiles", "rasterize_gaussians_simple",
              "bin_and_sort_gaussians", "compute_cumulative_intersects", "compute_cov2d_bounds",
              "get_tile_bin_edges", "map_gaussian_to_intersects"):
        assert callable(getattr(gsplat, n)), n


def test_cpu_tensors_rejected_like_reference():
    import torch
    from gsplat import csrc

    x = torch.zeros(4, 2)
    with pytest.raises(RuntimeError, match="gaussian_ids_sorted must be a CUDA tensor"):
        csrc.nd_rasterize_forward_topk_norm((1, 1, 1), (16, 16, 1), (16, 16, 1),
                                            torch.zeros(4, dtype=torch.int32),
                                            torch.zeros(1, 2, dtype=torch.int32), x,
                                            torch.zeros(4, 3), torch.zeros(4, 3))


def test_loss_and_multiview_check_arguments_before_any_launch():
    """The fused loss and the multi-view step reject bad arguments on the
    host, before anything reaches a GPU."""
    import torch

    import multiview
    from gsplat.loss import l2_loss_grad

    with pytest.raises(RuntimeError, match="pred must be a CUDA tensor"):
        l2_loss_grad(torch.zeros(8), torch.zeros(8))
    with pytest.raises(ValueError, match="streams must be >= 1"):
        multiview.ViewPipeline([torch.zeros(3)], streams=0)
    p = [torch.zeros(2)] * 7
    with pytest.raises(ValueError, match="params and grads"):
        multiview.fit_step_views(p[:6], [], [], torch.zeros(3), 10.0, p, torch.zeros(1))
    with pytest.raises(ValueError, match="one target per camera"):
        multiview.fit_step_views(p, [object()], [], torch.zeros(3), 10.0, p, torch.zeros(1))
    three = ([object()] * 3, [torch.zeros(3)] * 3)
    for group in (0, [2, 2], [3, 0], [1, 1]):
        with pytest.raises(ValueError, match="group"):
            multiview.fit_step_views(p, *three, torch.zeros(3), 10.0, p, torch.zeros(1),
                                     group=group)


def test_view_groups_split_a_ranks_views():
    """Balanced groups of at most `group` views and at most half of the
    views each (two streams, a group each); every view in exactly one."""
    from multiview import view_groups

    assert view_groups(64, 8) == [8] * 8
    assert view_groups(8, 8) == [4, 4]
    assert view_groups(9, 4) == [3, 3, 3]
    assert view_groups(1, 8) == [1] and view_groups(0, 8) == []
    for n in range(1, 70):
        for g in (1, 2, 3, 8):
            sizes = view_groups(n, g)
            assert sum(sizes) == n and min(sizes) >= 1 and max(sizes) <= max(1, g)
            assert max(sizes) - min(sizes) <= 1 and (n < 2 or len(sizes) >= 2)


def test_geometry_backward_rejects_misaligned_buffers():
    """The geometry backward reads rotations as float4 and scales as float2:
    a buffer that does not start on that boundary is rejected by the C-ABI
    before any launch (fake addresses; nothing is dereferenced)."""
    from gsplat._lib import lib

    ok16, ok8, bad16, bad8 = 0x10000, 0x20000, 0x30008, 0x40004
    fn = lib.dll.hx_hexels3d_geometry_backward

    def call(scales, rotations, grad_scales, grad_rotations):
        return fn(1, 1, ok16, scales, 1.0, rotations, ok16, ok16, 8, 8, ok16, ok16, ok16, ok16,
                  None, None, ok16, None, 3, grad_scales, grad_rotations, 1, None)

    for args in ((ok8, bad16, ok8, ok16), (ok8, ok16, ok8, bad16), (bad8, ok16, ok8, ok16),
                 (ok8, ok16, bad8, ok16)):
        assert call(*args) != 0
        assert b"boundary" in lib.dll.hx_last_error()


def test_topk_backward_rows_rejects_bad_ranges():
    """The stripe backward checks 0 <= begin <= end <= H before any launch
    (fake addresses; nothing is dereferenced); an empty range is a no-op."""
    from gsplat._lib import lib

    a = 0x10000
    fn = lib.dll.hx_nd_rasterize_backward_topk_norm_rows

    def call(r0, r1):
        return fn(64, 48, 3, 10, a, a, a, a, None, None, a, r0, r1, a, a, a, None)

    for r0, r1 in ((-16, 16), (32, 16), (0, 64)):
        assert call(r0, r1) != 0
        assert b"rows must satisfy" in lib.dll.hx_last_error()
    assert call(16, 16) == 0


def test_tensors_on_another_device_are_rejected():
    """Raw pointers run on the first tensor's device, so a tensor on another
    device is rejected on the host (metadata only: cpu against meta)."""
    import torch

    from gsplat._lib import check_same_device

    a = torch.zeros(4)
    check_same_device(a, "pred", target=torch.zeros(4), grad=None)
    with pytest.raises(RuntimeError, match="target is on meta but pred is on cpu"):
        check_same_device(a, "pred", target=torch.zeros(4, device="meta"))


def test_packaged_abi_table_matches_the_header():
    """The loader binds gsplat/_abi_table.py (written by the build), so an
    installed package reads no header: the table must be the header's."""
    import importlib.util

    pkg = os.path.join(ROOT, "hexel-kernel_b200", "gsplat")
    spec = importlib.util.spec_from_file_location("_hx_abi", os.path.join(pkg, "_abi.py"))
    abi = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(abi)
    from gsplat._abi_table import SIGNATURES

    parsed = abi.parse_header(HEADER)
    assert {k: (r, list(a)) for k, (r, a) in SIGNATURES.items()} == parsed
    assert set(parsed) == set(declared())
