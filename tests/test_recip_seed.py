"""The sigmoid epilogue's reciprocal seed constant (CPU).

The pointwise sigmoid kind takes 1 / (1 + 2^t) on the FMA pipe from a bit-level
initial guess and Newton steps (one for a bf16 P, with a centring output scale;
two for fp16). These tests check that the constant in the
CUDA source is the one ``recip_seed.py`` derives (a local optimum of the seed's
largest relative error over every mantissa), and that the resulting reciprocal
is accurate far beyond the 16-bit P it feeds.
"""
import os
import re

import numpy as np

from chia_proj_b200.csrc import recip_seed as rs

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "..", "chia_proj_b200", "csrc", "fmha_sm100.cuh")


def test_source_uses_the_derived_constant():
    text = open(SRC).read()
    # the kernel subtracts from the sign-flipped constant (it works on -y)
    found = set(int(m, 16) for m in re.findall(r"0x(FEF311[0-9A-F]{2})u", text))
    assert found == {rs.KERNEL_SEED | 0x80000000}


def test_constant_is_a_local_optimum():
    e0 = rs.seed_error(rs.KERNEL_SEED)
    assert 0.0505 < e0 < 0.0506
    for d in (-8, -3, -1, 1, 3, 8):
        assert rs.seed_error(rs.KERNEL_SEED + d) >= e0


def test_centring_scale_in_source_and_one_step_error():
    """bf16 P: one Newton step, the output scaled by 1 / (1 - e0^2 / 2)."""
    text = open(SRC).read()
    m = re.search(r"kSigmoidCentre = ([0-9.]+)f;", text)
    assert m is not None
    scale = float(m.group(1))
    assert abs(scale - rs.centre_scale()) < 1e-9
    rng = np.random.default_rng(1)
    t = np.concatenate([rng.uniform(-30, 30, 200_000), np.array([-30.0, 0.0, 1.0, 30.0])])
    y = (1.0 + np.exp2(t)).astype(np.float32)
    r = rs.sigmoid_recip(y, steps=1).astype(np.float64) * scale
    rel = np.abs(r * y.astype(np.float64) - 1.0)
    half = rs.seed_error(rs.KERNEL_SEED) ** 2 / 2
    assert rel.max() < half + 2e-6
    assert rel.max() < 2.0 ** -9  # below the rounding of a bf16 P


def test_reciprocal_error_after_two_newton_steps():
    rng = np.random.default_rng(0)
    # y = 1 + 2^t over the range the epilogue produces (t clamped at 126)
    t = np.concatenate([rng.uniform(-30, 30, 200_000), rng.uniform(30, 120, 20_000),
                        np.array([-30.0, 0.0, 1.0, 120.0])])
    y = (1.0 + np.exp2(t)).astype(np.float32)
    r = rs.sigmoid_recip(y).astype(np.float64)
    rel = np.abs(r * y.astype(np.float64) - 1.0)
    assert rel.max() < 2e-6 + rs.seed_error(rs.KERNEL_SEED) ** 4
    # near the clamp the seed falls below the normal range and loses digits;
    # the result (about 1e-38) is still far inside the 16-bit rounding of P
    t = np.linspace(120.0, 126.0, 10_000)
    y = (1.0 + np.exp2(t)).astype(np.float32)
    r = rs.sigmoid_recip(y).astype(np.float64)
    rel = np.abs(r * y.astype(np.float64) - 1.0)
    assert rel.max() < 2.0 ** -9 / 16
