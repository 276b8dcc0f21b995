"""CPU oracle for the ten attention variants -- TEST INFRASTRUCTURE ONLY.

This package is a checker, never a product path. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it. The library in ``chia_proj_b200`` never
imports it and has no CPU fallback.

``oracle.eager`` restates, in fp32 PyTorch on the CPU, the eager reference
functions of JoshiP-commits/CHIA_proj (``extra_bench.py:32-62`` and the
corrected sigmoid reference ``sigmoid_fix.py:34-40``), generalised with the
parameters the benchmark configurations use (softcap value, window, block,
prefix, dilation, ALiBi slopes, per-head temperatures, sigmoid bias, ReLU
output scale). With default arguments every function computes exactly the
reference's formula.

Parity of this restatement is pinned against golden vectors produced by
executing the reference's own ``build_refs`` / ``ref_sigmoid`` source on the
CPU (``tests/golden/make_golden.py``); ``tests/test_oracle.py`` checks it.
"""

from .eager import (  # noqa: F401
    OPS,
    reference_masks,
    run_op,
    run_op_lse,
    run_varlen,
    visible_pairs_dense,
)
