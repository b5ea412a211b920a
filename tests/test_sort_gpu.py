"""The radix sort (hx_sort_pairs_u32 / _u64) against numpy's stable sort:
keys and values bit-exact (stable order of equal keys), for sizes on both
sides of the 4-keys / 16-keys-per-thread tile switch (2M keys), one to eight
8-bit passes, ragged tails, many equal keys."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _sort(keys: torch.Tensor, begin_bit: int, end_bit: int):
    from gsplat._lib import lib, ptr, stream, workspace

    n = keys.numel()
    dev = keys.device
    vals = torch.arange(n, dtype=torch.int32, device=dev)
    ko = torch.empty_like(keys)
    vo = torch.empty_like(vals)
    kb = keys.element_size()
    ws = workspace(lib.query("hx_sort_pairs_workspace_bytes", n, kb), dev)
    name = "hx_sort_pairs_u64" if kb == 8 else "hx_sort_pairs_u32"
    lib.call(name, ptr(keys), ptr(vals), ptr(ko), ptr(vo), n, begin_bit, end_bit, ptr(ws),
             ws.numel(), stream(dev))
    return ko, vo


@pytest.mark.parametrize("n,bits,distinct", [
    (1, 8, 256), (1000, 13, 8192), (4097, 32, 2**32), (300_001, 20, 50),
    (1_000_000, 32, 2**32), (2_100_003, 13, 8160), (3_531_440, 13, 8160),
])
def test_sort_u32_matches_stable_numpy(n, bits, distinct):
    g = torch.Generator().manual_seed(n)
    keys = torch.randint(0, min(distinct, 2**bits), (n,), generator=g, dtype=torch.int64)
    keys32 = keys.to(torch.int32)  # reinterpreted as uint32 by the library
    ko, vo = _sort(keys32.cuda(), 0, bits)
    k_np = keys.numpy().astype(np.uint32)
    order = np.argsort(k_np, kind="stable")
    assert np.array_equal(ko.cpu().numpy().astype(np.uint32), k_np[order])
    assert np.array_equal(vo.cpu().numpy(), order.astype(np.int32))


@pytest.mark.parametrize("n,end_bit", [(37, 40), (65_537, 45), (2_500_000, 64)])
def test_sort_u64_matches_stable_numpy(n, end_bit):
    g = torch.Generator().manual_seed(7 + n)
    tile = torch.randint(0, 8160, (n,), generator=g, dtype=torch.int64)
    low = torch.randint(0, 2**31, (n,), generator=g, dtype=torch.int64)
    keys = (tile << 32) | low
    if end_bit < 64:
        keys = keys & ((1 << end_bit) - 1)
    ko, vo = _sort(keys.cuda(), 0, end_bit)
    k_np = keys.numpy().view(np.uint64)
    order = np.argsort(k_np, kind="stable")
    assert np.array_equal(ko.cpu().numpy().view(np.uint64), k_np[order])
    assert np.array_equal(vo.cpu().numpy(), order.astype(np.int32))
