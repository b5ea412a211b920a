"""Build recipe for the reference rasteriser, used only as a test checker.

This is test infrastructure.  It compiles the reference project's CUDA
sources *where they lie* (``gsplat/cuda/csrc`` and ``gsplat/cuda_hexels3d/csrc``
of honeycomb-surfels/hexel-kernel) into ``oracle/_ref/`` with the reference's
own compiler flags (``-O3 --use_fast_math --expt-relaxed-constexpr``,
reference ``setup.py:88-100``) for sm_100a.  Nothing is copied into the
repository and the reference's own ``setup.py`` is not run.

The two resulting Python extension modules are named ``_ref_gsplat_csrc`` and
``_ref_hexels3d_C`` so that they never collide with this repository's
``gsplat`` package.  GPU parity tests import them (when present) to compare
the B200 kernels bit-for-bit (binning, sort, ranges, top-K ids) and within
tolerance (images, gradients) against the reference on identical inputs.

Usage::

    python oracle/build_ref.py --reference DIR [--jobs N]

(or HEXEL_REFERENCE_DIR=DIR in the environment).

The reference tree is only needed when building; the built ``.so`` files
travel with the repository snapshot.
"""

from __future__ import annotations

import argparse
import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")

REF_FLAGS = ["-O3", "--use_fast_math", "--expt-relaxed-constexpr"]
ARCH = ["-gencode=arch=compute_100a,code=sm_100a"]


def _build(name: str, sources: list[str], include: list[str], jobs: int) -> str:
    from torch.utils import cpp_extension

    build_dir = os.path.join(OUT, "build_" + name)
    os.makedirs(build_dir, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(jobs))
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    mod = cpp_extension.load(
        name=name,
        sources=sources,
        extra_include_paths=include,
        extra_cflags=["-O3", "-Wno-sign-compare"],
        extra_cuda_cflags=REF_FLAGS + ARCH,
        build_directory=build_dir,
        with_cuda=True,
        verbose=False,
    )
    so = mod.__file__
    dst = os.path.join(OUT, os.path.basename(so))
    if os.path.abspath(so) != os.path.abspath(dst):
        import shutil

        shutil.copy2(so, dst)
    return dst


def build(reference: str, jobs: int = 8) -> list[str]:
    if not os.path.isdir(reference):
        raise FileNotFoundError(f"reference tree not found at {reference}")
    os.makedirs(OUT, exist_ok=True)
    csrc = os.path.join(reference, "gsplat", "cuda", "csrc")
    glm = os.path.join(csrc, "third_party", "glm")
    h3d = os.path.join(reference, "gsplat", "cuda_hexels3d", "csrc")
    built = []
    srcs2d = sorted(glob.glob(os.path.join(csrc, "*.cu")) + glob.glob(os.path.join(csrc, "*.cpp")))
    built.append(_build("_ref_gsplat_csrc", srcs2d, [csrc, glm], jobs))
    srcs3d = sorted(glob.glob(os.path.join(h3d, "*.cu")) + glob.glob(os.path.join(h3d, "*.cpp")))
    built.append(_build("_ref_hexels3d_C", srcs3d, [h3d, glm], jobs))
    return built


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HEXEL_REFERENCE_DIR"),
                    help="the reference project's source tree (or HEXEL_REFERENCE_DIR)")
    ap.add_argument("--jobs", type=int, default=8)
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference DIR or set HEXEL_REFERENCE_DIR")
    for path in build(args.reference, args.jobs):
        print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
