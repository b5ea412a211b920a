"""Loader of ``libhexel_b200.so`` — the C-ABI declared in ``include/hexel_b200.h``.

The Python host code in this package calls the CUDA kernels only through this
module.  Pointers are raw device addresses (``Tensor.data_ptr()``), the stream
is PyTorch's current stream on the tensors' device, and a non-zero status is
raised as ``RuntimeError`` carrying the library's message.  There is no
fallback: if the library is missing or was built for a different ABI version,
importing this module fails.
"""

from __future__ import annotations

import ctypes
import math
import os
import re
from typing import Optional

import torch

ABI_VERSION = 1
_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhexel_b200.so")

_RET = {"int": ctypes.c_int, "size_t": ctypes.c_size_t, "const char*": ctypes.c_char_p,
        "void": None, "unsigned long long": ctypes.c_ulonglong}
_ARG = {"ptr": ctypes.c_void_p, "int": ctypes.c_int, "unsigned": ctypes.c_uint,
        "float": ctypes.c_float, "size_t": ctypes.c_size_t, "int32_t": ctypes.c_int32,
        "int64_t": ctypes.c_int64}


def _ctypes_signatures(table: dict) -> dict:
    return {name: (_RET[ret], [_ARG[k] for k in args]) for name, (ret, args) in table.items()}


class _Lib:
    def __init__(self, path: str):
        if not os.path.exists(path):
            raise ImportError(
                f"{path} is missing: build the CUDA library with "
                "`python hexel-kernel_b200/build.py` (or __graft_entry__.build())."
            )
        self.path = path
        self.dll = ctypes.CDLL(path)
        from ._abi_table import SIGNATURES

        self.signatures = _ctypes_signatures(SIGNATURES)
        for name, (res, args) in self.signatures.items():
            fn = getattr(self.dll, name)
            fn.restype = res
            fn.argtypes = args
        ver = self.dll.hx_abi_version()
        if ver != ABI_VERSION:
            raise ImportError(f"{path} has ABI version {ver}, expected {ABI_VERSION}; rebuild it")

    def call(self, name: str, *args) -> None:
        rc = getattr(self.dll, name)(*args)
        if rc != 0:
            msg = self.dll.hx_last_error().decode(errors="replace")
            raise RuntimeError(f"{name} failed ({rc}): {msg}")

    def query(self, name: str, *args) -> int:
        return int(getattr(self.dll, name)(*args))


lib = _Lib(_LIB_PATH)


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    """Device address of a tensor, or None (NULL) for an absent one."""
    if t is None:
        return None
    return t.data_ptr()


def stream(device: torch.device) -> int:
    """The current CUDA stream of `device` as a raw cudaStream_t."""
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Caller-owned scratch memory from PyTorch's caching allocator."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def zero_views(device: torch.device, shapes) -> list:
    """Zero-filled float32 tensors of the given shapes carved out of one
    allocation (one fill launch instead of one per tensor); each view starts
    on a 16-byte boundary so the kernels' vector loads stay aligned."""
    sizes = [int(math.prod(s)) for s in shapes]
    padded = [(n + 3) // 4 * 4 for n in sizes]
    buf = torch.zeros(max(1, sum(padded)), dtype=torch.float32, device=device)
    out, o = [], 0
    for shape, n, pn in zip(shapes, sizes, padded):
        out.append(buf[o:o + n].view(shape))
        o += pn
    return out


def check_same_device(ref: torch.Tensor, ref_name: str, **others) -> None:
    """Raises RuntimeError unless every tensor in `others` (name=tensor, None
    allowed) lives on `ref`'s device: the kernels take raw pointers and run
    on `ref`'s device, where another GPU's address would be invalid."""
    for name, t in others.items():
        if t is not None and t.device != ref.device:
            raise RuntimeError(f"{name} is on {t.device} but {ref_name} is on {ref.device}")


def check_input(t: torch.Tensor, name: str) -> None:
    """Mirrors the reference's CHECK_INPUT (gsplat/cuda/csrc/bindings.h:10-15)."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
