"""Mask geometry and the kernel's key-tile schedule, checked without a GPU.

The library's integer mask model (``include/chia_attn.h``) must reproduce the
reference's boolean masks (``extra_bench.py:55-61``) pair for pair, and the
tile plan the kernel executes must cover every visible pair and only skip
the element-wise mask on tiles that are completely visible.
"""

import itertools
import random

import pytest
import torch

import chia_proj_b200 as cp
from oracle.eager import reference_masks


def dense(mask: cp.Mask, sq: int, skv: int) -> torch.Tensor:
    """Dense boolean visibility straight from the header's definition."""
    i = torch.arange(sq).view(-1, 1)
    j = torch.arange(skv).view(1, -1)
    band = torch.ones(sq, skv, dtype=torch.bool)
    if mask.left >= 0:
        band &= (i - j) <= mask.left
    if mask.right >= 0:
        band &= (j - i) <= mask.right
    if mask.block > 0:
        band &= torch.div(i, mask.block, rounding_mode="floor") == \
            torch.div(j, mask.block, rounding_mode="floor")
    band &= ((i - j) % mask.dilation) == 0
    return band | (j < mask.prefix)


REF_CASES = [
    ("bias_sliding_window", dict(window=256), dict()),
    ("bias_local", dict(window=256), dict()),
    ("bias_block_diagonal", dict(block=512), dict()),
    ("bias_dilated", dict(dilation=4), dict()),
    ("bias_prefix_lm", dict(prefix=256), dict()),
]


@pytest.mark.parametrize("S", [1, 7, 255, 256, 257, 544, 1000])
@pytest.mark.parametrize("op,kw,_", REF_CASES)
def test_op_masks_equal_reference_masks(lib, op, kw, _, S):
    ref = reference_masks()[op]
    i = torch.arange(S).view(-1, 1)
    j = torch.arange(S).view(1, -1)
    assert torch.equal(dense(cp.op_config(op, **kw), S, S), ref(i, j))
    assert cp.visible_pairs(cp.op_config(op, **kw), S) == int(ref(i, j).sum())


def test_causal_and_full(lib):
    for S in (1, 2, 129, 640):
        assert cp.visible_pairs(cp.CAUSAL, S) == S * (S + 1) // 2
        assert cp.visible_pairs(cp.FULL, S) == S * S


def _random_masks(n, seed=0):
    rnd = random.Random(seed)
    out = []
    for _ in range(n):
        out.append(cp.Mask(left=rnd.choice([-1, 0, 1, 5, 100, 255, 300]),
                           right=rnd.choice([-1, 0, 3, 127, 200]),
                           block=rnd.choice([0, 0, 64, 100, 256]),
                           prefix=rnd.choice([0, 0, 1, 130, 1000]),
                           dilation=rnd.choice([1, 1, 2, 3, 4])))
    return out


@pytest.mark.parametrize("mask", _random_masks(40))
def test_visible_pairs_random(lib, mask):
    for sq, skv in ((300, 300), (513, 513), (200, 260)):
        assert cp.visible_pairs(mask, sq, skv) == int(dense(mask, sq, skv).sum()), (mask, sq, skv)


@pytest.mark.parametrize("mask", _random_masks(40, seed=1) + [cp.op_config(o, **k)
                                                             for o, k, _ in REF_CASES])
def test_tile_plan_covers_and_full_tiles_are_full(lib, mask):
    """Every visible pair lies in a visited tile; 'full' tiles are completely visible."""
    BM = BN = 128
    for S in (300, 700):
        vis = dense(mask, S, S)
        for row0 in range(0, S, BM):
            lo, hi, bits = cp.tile_plan(mask, S, row0, BM, BN)
            rows = vis[row0:row0 + BM]
            cols_needed = rows.any(0).nonzero().flatten()
            if cols_needed.numel():
                assert lo * BN <= int(cols_needed.min()) and int(cols_needed.max()) < hi * BN
            for t in range(lo, hi):
                blk = rows[:, t * BN:(t + 1) * BN]
                complete = blk.shape[1] == BN and bool(blk.all())
                if bits >> (t - lo) & 1:
                    assert complete, (mask, S, row0, t)
                elif mask.dilation == 1 and mask.prefix == 0 and t - lo < 64:
                    # without a prefix a completely visible tile lies in every
                    # row's band, which the plan must recognise
                    assert not complete, ("missed full tile", mask, S, row0, t)


def test_reference_masks_skip_work(lib):
    """Banded masks visit only the band: a 256 window touches 3 of 32 tiles per row tile."""
    S = 4096
    lo, hi, bits = cp.tile_plan(cp.op_config("bias_sliding_window"), S, 2048)
    assert (lo, hi) == (14, 17)
    lo, hi, bits = cp.tile_plan(cp.op_config("bias_block_diagonal", block=256), S, 2048 + 128)
    assert (lo, hi) == (16, 18)   # only the current block
    lo, hi, _ = cp.tile_plan(cp.CAUSAL, S, 0)
    assert (lo, hi) == (0, 1)


def test_flop_counts_of_the_benchmark_configs(lib):
    """Mask-aware FLOPs of the BASELINE configurations (4*D*pairs*B*H)."""
    assert cp.visible_pairs(cp.op_config("bias_sliding_window"), 2048) == 491648
    assert cp.visible_pairs(cp.CAUSAL, 4096) == 8390656
    assert cp.visible_pairs(cp.op_config("bias_prefix_lm", prefix=1024), 4096) == 8914432
    assert cp.visible_pairs(cp.op_config("bias_block_diagonal", block=256), 4096) == 526336
    assert cp.visible_pairs(cp.op_config("bias_dilated", dilation=4), 4096) == 2099200
    assert cp.visible_pairs(cp.op_config("bias_local"), 4096) == 2027776
    assert cp.visible_pairs(cp.FULL, 8192) == 67108864
    f = cp.mask_aware_flops(cp.FULL, 32, 32, 8192, 128)
    assert abs(f / 1e12 - 35.18) < 0.01
