"""The flex_attention-compatible frontend (chia_proj_b200/flex.py).

The callables are the reference's own flex specification of eight operators
(JoshiP-commits/CHIA_proj extra_bench.py:85-95): mask_mods are fitted to the
library's mask model and checked element by element, score_mods are
identified by evaluation. CPU tests cover the fitting; GPU tests run
flex_attention against the fp32 oracle.
"""

import math

import pytest
import torch

import chia_proj_b200 as cp
from chia_proj_b200 import flex
import oracle

H = 4
SLOPES = torch.arange(1, H + 1, dtype=torch.float32)
TEMPS = 0.5 + torch.arange(H, dtype=torch.float32) / H
causal = lambda b, h, qi, kj: kj <= qi
REF_FLEX = {
    "temp_perhead": (lambda sc, b, h, qi, kj: sc * TEMPS[h], causal),
    "bias_alibi": (lambda sc, b, h, qi, kj: sc + SLOPES[h] * (kj - qi), causal),
    "softcap_gemma2": (lambda sc, b, h, qi, kj: torch.tanh(sc / 30.0) * 30.0, causal),
    "bias_dilated": (None, lambda b, h, qi, kj: (kj <= qi) & (((qi - kj) % 4) == 0)),
    "bias_local": (None, lambda b, h, qi, kj: (qi - kj).abs() < 256),
    "bias_block_diagonal": (None, lambda b, h, qi, kj: ((qi // 512) == (kj // 512)) & (kj <= qi)),
    "bias_prefix_lm": (None, lambda b, h, qi, kj: (kj <= qi) | (kj < 256)),
    "bias_sliding_window": (None, lambda b, h, qi, kj: (kj <= qi) & ((qi - kj) < 256)),
}


@pytest.mark.parametrize("op", sorted(REF_FLEX))
@pytest.mark.parametrize("S", [300, 1100])
def test_reference_mask_mods_fit_the_operator_masks(op, S):
    _, mask_mod = REF_FLEX[op]
    bm = flex.create_block_mask(mask_mod, B=None, H=None, Q_LEN=S, KV_LEN=S, device="cpu")
    want = cp.op_config(op) if op not in ("temp_perhead", "bias_alibi", "softcap_gemma2") \
        else cp.CAUSAL
    # the fit is exact on the grid; for the reference parameters it is the operator's mask
    # (a prefix or window wider than S may fit as an equivalent simpler mask)
    i = torch.arange(S)
    assert torch.equal(flex._mask_dense(bm.mask, i, S), flex._mask_dense(want, i, S))
    assert torch.equal(flex._mask_dense(bm.mask, i, S), mask_mod(0, 0, i.view(-1, 1), i.view(1, -1)))


def test_fitted_masks_are_the_kernel_parameters():
    S = 4096
    fit = lambda f: flex.create_block_mask(f, None, None, S, S, device="cpu").mask
    assert fit(causal) == cp.Mask(left=-1, right=0)
    assert fit(REF_FLEX["bias_sliding_window"][1]) == cp.Mask(left=255, right=0)
    assert fit(REF_FLEX["bias_local"][1]) == cp.Mask(left=255, right=255)
    assert fit(REF_FLEX["bias_block_diagonal"][1]) == cp.Mask(left=-1, right=0, block=512)
    assert fit(REF_FLEX["bias_dilated"][1]) == cp.Mask(left=-1, right=0, dilation=4)
    assert fit(REF_FLEX["bias_prefix_lm"][1]) == cp.Mask(left=-1, right=0, prefix=256)
    assert fit(lambda b, h, qi, kj: kj >= 0) == cp.Mask(left=-1, right=-1)
    # decode-shaped, bottom-right causal
    bm = flex.create_block_mask(lambda b, h, qi, kj: kj <= qi + 900, None, None, 100, 1000,
                                device="cpu")
    assert bm.mask == cp.Mask(left=-1, right=900)


def test_large_masks_are_checked_on_sampled_rows():
    S = 16384   # 2^28 entries: evaluated on a sample of rows
    bm = flex.create_block_mask(REF_FLEX["bias_sliding_window"][1], None, None, S, S,
                                device="cpu")
    assert bm.mask == cp.Mask(left=255, right=0)


@pytest.mark.parametrize("mask_mod", [
    lambda b, h, qi, kj: (kj < qi),                       # strictly causal: right would be -1
    lambda b, h, qi, kj: ((qi + kj) % 3) == 0,            # stride 3, but j = -i (mod 3)
    lambda b, h, qi, kj: (kj <= qi) & (h == 0) | (kj <= qi - 5),  # depends on the head
])
def test_masks_without_a_counterpart_are_rejected(mask_mod):
    with pytest.raises(flex.NotExpressible):
        flex.create_block_mask(mask_mod, B=2, H=3, Q_LEN=200, KV_LEN=200, device="cpu")


def test_a_congruence_mask_fits_as_dilation():
    # (7 i + 3 j) % 5 == 0  <=>  (i - j) % 5 == 0: a full dilated mask
    bm = flex.create_block_mask(lambda b, h, qi, kj: ((qi * 7 + kj * 3) % 5) == 0, None, None,
                                300, 300, device="cpu")
    assert bm.mask == cp.Mask(left=-1, right=-1, dilation=5)


def test_score_mods_are_identified():
    ident = lambda sm: flex.identify_score_mod(sm, H, "cpu")
    assert ident(None).mod == "none"
    assert ident(lambda sc, b, h, qi, kj: sc).mod == "none"
    t = ident(REF_FLEX["temp_perhead"][0])
    assert t.mod == "temp" and torch.allclose(t.head_param, TEMPS)
    a = ident(REF_FLEX["bias_alibi"][0])
    assert a.mod == "alibi" and torch.allclose(a.head_param, SLOPES)
    c = ident(REF_FLEX["softcap_gemma2"][0])
    assert c.mod == "softcap" and abs(c.softcap - 30.0) < 1e-3
    with pytest.raises(flex.NotExpressible):
        ident(lambda sc, b, h, qi, kj: 2 * sc + 1)
    with pytest.raises(flex.NotExpressible):  # softcap and ALiBi together
        ident(lambda sc, b, h, qi, kj: torch.tanh(sc / 30) * 30 + SLOPES[h] * (kj - qi))


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
@pytest.mark.parametrize("op", sorted(REF_FLEX))
def test_flex_attention_matches_the_oracle(cuda, op):
    """flex_attention(q, k, v, score_mod, block_mask) with the reference's
    callables, against the reference operator (fp32 oracle)."""
    S, D = 1000, 128
    g = torch.Generator().manual_seed(13)
    q, k, v = (torch.randn(1, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    score_mod, mask_mod = REF_FLEX[op]
    # as in the reference, the per-head parameters the callables capture live
    # on the device the call runs on
    sl, te = SLOPES.to(cuda), TEMPS.to(cuda)
    score_mod = {"temp_perhead": lambda sc, b, h, qi, kj: sc * te[h],
                 "bias_alibi": lambda sc, b, h, qi, kj: sc + sl[h] * (kj - qi)}.get(op, score_mod)
    bm = flex.create_block_mask(mask_mod, None, None, S, S, device=cuda)
    out = flex.flex_attention(q.to(cuda), k.to(cuda), v.to(cuda), score_mod=score_mod,
                              block_mask=bm)
    torch.cuda.synchronize()
    ref = oracle.run_op(op, q, k, v)
    err = (out.float().cpu() - ref).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, op


@pytest.mark.gpu
def test_flex_attention_gqa_and_lse(cuda):
    S, D, Hkv = 700, 64, 2
    g = torch.Generator().manual_seed(14)
    q = torch.randn(1, H, S, D, generator=g).to(torch.bfloat16)
    k, v = (torch.randn(1, Hkv, S, D, generator=g).to(torch.bfloat16) for _ in range(2))
    bm = flex.create_block_mask(causal, None, None, S, S, device=cuda)
    out, lse = flex.flex_attention(q.to(cuda), k.to(cuda), v.to(cuda), block_mask=bm,
                                   enable_gqa=True, return_lse=True)
    torch.cuda.synchronize()
    kr, vr = (x.repeat_interleave(H // Hkv, dim=1) for x in (k, v))
    ref, ref_lse = oracle.run_op_lse("bias_dilated", q, kr, vr, dilation=1)
    assert (out.float().cpu() - ref).abs().max().item() < 2e-2
    assert (lse.cpu() - ref_lse).abs().max().item() < 1e-3
