"""Plugin module for the reference's kernel loader: ``bias_dilated``.

JoshiP-commits/CHIA_proj discovers ``*_BEST.py`` files and calls their
``launch_kernel(q, k, v)`` (loader ``extra_bench.py:24-27``, discovery
``extra_bench.py:65-70``). This module keeps that contract, with the
reference's default parameters, and runs the sm_100a kernel of
``chia_proj_b200``.
"""
import os as _os
import sys as _sys

_ROOT = _os.path.dirname(_os.path.dirname(_os.path.dirname(_os.path.realpath(__file__))))
if _ROOT not in _sys.path:
    _sys.path.insert(0, _ROOT)

from chia_proj_b200 import bias_dilated as _op  # noqa: E402


def launch_kernel(q, k, v):
    return _op(q, k, v)
