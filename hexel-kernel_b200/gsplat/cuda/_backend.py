"""Binds the 2D extension module (``gsplat.csrc``), as the reference's
gsplat/cuda/_backend.py:1-13 does.  Importing fails loudly if the CUDA
library is missing; there is no fallback."""

try:
    from gsplat import csrc as _C
except ImportError as error:
    raise ImportError(
        "Cannot load the B200 rasteriser library behind `gsplat.csrc`; build it with "
        "`python hexel-kernel_b200/build.py`."
    ) from error

__all__ = ["_C"]
