"""Generate golden vectors by executing the reference's own eager functions.

Run in a container that has the reference checkout (read-only) available::

    python tests/golden/make_golden.py --reference <path-to-CHIA_proj>

The reference scripts cannot be imported as modules (they allocate CUDA
tensors and open network clients at import time), so this script parses them
with ``ast`` and executes only two function definitions, unchanged, in a
namespace where ``dev="cpu"`` and ``DT=torch.float32``:

* ``build_refs(S)`` from ``extra_bench.py:32-62`` -- the ten eager operators;
* ``ref_sigmoid(q, k, v)`` from ``sigmoid_fix.py:34-40`` -- the corrected
  sigmoid reference.

The module-level constants those functions read (``D``, ``H``, ``S``, ``SC``)
are set to the fixture shape. Inputs are seeded N(0,1) draws rounded to bf16
(so the same values feed the bf16 GPU kernel), then the reference functions
run on their fp32 upcast. Output: ``tests/golden/reference_B1H2S544D64.pt``.
"""

from __future__ import annotations

import argparse
import ast
import math
import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
B, H, S, D = 1, 2, 544, 64       # S > 512 so block 512 / window 256 / prefix 256 all bite
SEED = 1234


def _extract(path: str, names):
    """Return the source of the named top-level function definitions in ``path``."""
    with open(path) as fh:
        src = fh.read()
    tree = ast.parse(src)
    out = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            out.append(ast.get_source_segment(src, node))
    missing = set(names) - {n.name for n in tree.body if isinstance(n, ast.FunctionDef)}
    if missing:
        raise RuntimeError(f"{path}: functions not found: {sorted(missing)}")
    return "\n\n".join(out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the CHIA_proj checkout")
    ap.add_argument("--out", default=os.path.join(HERE, f"reference_B{B}H{H}S{S}D{D}.pt"))
    a = ap.parse_args()

    ns = {"torch": torch, "F": F, "math": math, "dev": "cpu",
          "DT": torch.float32, "H": H, "D": D, "S": S, "SC": 1.0 / math.sqrt(D)}
    exec(compile(_extract(os.path.join(a.reference, "extra_bench.py"), ["build_refs"]),
                 "extra_bench.py::build_refs", "exec"), ns)
    exec(compile(_extract(os.path.join(a.reference, "sigmoid_fix.py"), ["ref_sigmoid"]),
                 "sigmoid_fix.py::ref_sigmoid", "exec"), ns)

    g = torch.Generator().manual_seed(SEED)
    q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    qf, kf, vf = q.float(), k.float(), v.float()

    refs = ns["build_refs"](S)
    outs = {}
    with torch.no_grad():
        for op, fn in refs.items():
            outs[op] = fn(qf, kf, vf).float().contiguous()
        outs["sigmoid_fix.ref_sigmoid"] = ns["ref_sigmoid"](qf, kf, vf).float().contiguous()

    torch.save({"shape": (B, H, S, D), "seed": SEED, "q": q, "k": k, "v": v,
                "outputs": outs,
                "source": {"build_refs": "extra_bench.py:32-62",
                           "ref_sigmoid": "sigmoid_fix.py:34-40"}}, a.out)
    print(f"wrote {a.out}: {sorted(outs)}")


if __name__ == "__main__":
    sys.exit(main())
