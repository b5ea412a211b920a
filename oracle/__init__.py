"""CPU restatement of the reference rasteriser's algorithms — TEST INFRASTRUCTURE.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``gsplat`` in ``hexel-kernel_b200/``) never
imports it and fails loudly when its CUDA library is missing.

Modules restate the reference (honeycomb-surfels/hexel-kernel) formula by
formula, citing file:line; they are vectorised PyTorch fp32 on the CPU (the
floating-point work) and numpy (the integer binning work).  The CPU uses
IEEE ``exp``/division where the reference's CUDA build uses fast-math
intrinsics, so floating-point results agree to tolerance, and integer outputs
(binning, sorted lists, tile ranges) are exact given identical inputs.

Parity pinning: the reference ships no tests, fixtures or golden vectors.
The restatement is pinned by (a) ``tests/golden/`` vectors recorded from the
reference's own CUDA kernels (compiled from its sources by
``oracle/build_ref.py`` into ``oracle/_ref/``) on seeded inputs on a B200,
generator ``tests/golden/make_golden.py``, which ``tests/test_golden.py``
checks this restatement against on the CPU; (b) fp64 finite-difference checks
of its backward passes; (c) on a GPU, comparison with those reference kernels
on identical inputs, including the benchmarked sizes.
"""
