"""hx_inclusive_scan_i32_noalloc (fixed device scratch, no allocation)
against hx_inclusive_scan_i32 (caller workspace), called through the C-ABI.

Two calls in a row on different sizes (the larger first, so the second call
reads a scratch array still holding the first call's partial sums), and the
size limit.  Outputs are integers: they must be identical.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_N = 16384 * 4096


def _scan_with_workspace(lib, x):
    from gsplat._lib import ptr, stream, workspace

    out = torch.empty_like(x)
    total = torch.zeros(1, dtype=torch.int64, device=x.device)
    ws = workspace(lib.query("hx_scan_workspace_bytes", x.numel()), x.device)
    lib.call("hx_inclusive_scan_i32", ptr(x), ptr(out), x.numel(), ptr(total), ptr(ws),
             ws.numel(), stream(x.device))
    return out, total


def _scan_noalloc(lib, x):
    from gsplat._lib import ptr, stream

    out = torch.empty_like(x)
    total = torch.full((1,), -1, dtype=torch.int64, device=x.device)
    lib.call("hx_inclusive_scan_i32_noalloc", ptr(x), ptr(out), x.numel(), ptr(total),
             stream(x.device))
    return out, total


def test_noalloc_scan_matches_workspace_scan_twice():
    from gsplat._lib import lib

    g = torch.Generator(device="cuda").manual_seed(5)
    sizes = (3_000_001, 70_001)
    for n in sizes:
        x = torch.randint(0, 9, (n,), generator=g, device="cuda", dtype=torch.int32)
        ref_out, ref_total = _scan_with_workspace(lib, x)
        out, total = _scan_noalloc(lib, x)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), n
        assert int(total.item()) == int(ref_total.item()) == int(x.sum().item()), n


def test_noalloc_scan_limits():
    from gsplat._lib import lib, ptr, stream

    x = torch.ones(1, dtype=torch.int32, device="cuda")
    total = torch.full((1,), 7, dtype=torch.int64, device="cuda")
    lib.call("hx_inclusive_scan_i32_noalloc", ptr(x), ptr(x), 0, ptr(total), stream(x.device))
    assert int(total.item()) == 0
    with pytest.raises(RuntimeError, match="exceeds the fixed scratch maximum"):
        lib.call("hx_inclusive_scan_i32_noalloc", ptr(x), ptr(x), MAX_N + 1, ptr(total),
                 stream(x.device))
