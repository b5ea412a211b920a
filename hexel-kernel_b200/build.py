"""Builds libhexel_b200.so — every CUDA kernel of the package — for sm_100a.

Each ``csrc/*.cu`` file is compiled to an object with nvcc (in parallel), then
linked into one shared library placed next to the ``gsplat`` package.  The
library exports only the C-ABI declared in ``include/hexel_b200.h``.

    python hexel-kernel_b200/build.py [--force] [--jobs N]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "gsplat", "libhexel_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3",
    "--use_fast_math",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _compile(src: str, obj: str, extra: list[str]) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr}")


ABI_TABLE = os.path.join(PKG, "gsplat", "_abi_table.py")


def write_abi_table() -> None:
    """gsplat/_abi_table.py from include/hexel_b200.h (the loader binds this
    table, so an installed package needs no header)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_hx_abi", os.path.join(PKG, "gsplat",
                                                                         "_abi.py"))
    abi = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(abi)
    text = abi.render_table(abi.parse_header(os.path.join(INCLUDE, "hexel_b200.h")))
    if not os.path.exists(ABI_TABLE) or open(ABI_TABLE).read() != text:
        with open(ABI_TABLE, "w") as f:
            f.write(text)


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    write_abi_table()
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = _deps()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src, *deps, __file__]):
            todo.append((src, obj))
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_compile, s, o, extra) for s, o in todo]
        for f in futs:
            f.result()
    if todo or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        # Shared cudart: the library then runs in the same CUDA runtime instance as
        # PyTorch (one current device per host thread, same streams), which the
        # autograd engine's worker threads rely on.
        cuda_lib = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "lib64")
        cmd = [nvcc(), "-shared", "-cudart", "shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-Xlinker", "-rpath", "-Xlinker", cuda_lib, "-o", tmp, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose_ptxas=args.ptxas_v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
