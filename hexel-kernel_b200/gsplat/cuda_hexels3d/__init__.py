"""The 3D hexel rasteriser module ``gsplat.cuda_hexels3d._C``.

Importing it checks, as the reference's loader does
(gsplat/cuda_hexels3d/__init__.py:8-92), that the forward and backward entry
points exist with the expected argument counts (read from their
pybind-style signature docstrings), so stale builds are rejected loudly.
"""

from __future__ import annotations

import re
from typing import Any

from . import _C

_FWD_TENSORS, _FWD_TOTAL = 15, 27
_BWD_TENSORS, _BWD_TOTAL, _BWD_RETURNS = 21, 34, 12


def _arity(doc: str):
    tensors = len(re.findall(r"arg\d+:\s*torch\.Tensor", doc))
    total = len(re.findall(r"arg\d+:", doc))
    m = re.search(r"->\s*tuple\[(.*?)\]", doc, flags=re.DOTALL)
    returns = None if m is None else len(re.findall(r"torch\.Tensor", m.group(1)))
    return tensors, total, returns


def _validate(ext: Any) -> None:
    fw = getattr(ext, "rasterize_hexels3d_forward", None)
    bw = getattr(ext, "rasterize_hexels3d_backward", None)
    if fw is None or bw is None:
        raise ImportError("Missing expected Hexels3D rasterizer symbols.")
    ft, fa, _ = _arity(fw.__doc__ or "")
    bt, ba, br = _arity(bw.__doc__ or "")
    if (ft, fa) != (_FWD_TENSORS, _FWD_TOTAL):
        raise ImportError(f"Hexels3D module is out of date: forward takes {ft}/{fa} args")
    if (bt, ba) != (_BWD_TENSORS, _BWD_TOTAL) or (br is not None and br != _BWD_RETURNS):
        raise ImportError(f"Hexels3D module is out of date: backward takes {bt}/{ba} args")


_validate(_C)

__all__ = ["_C"]
