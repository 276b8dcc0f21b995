"""Backward pass (chia_attn_bwd) against autograd through the fp32 oracle.

The reference is forward only; the gradients checked here are those of its
eager functions (restated in oracle/eager.py) differentiated exactly by
torch.autograd in fp32 on the CPU. The kernel rounds P and dS to the input
type for the tensor cores (as the forward rounds P), so the bound is the
reference gate's relative form, max|g - g_ref| / max|g_ref| < 3e-2, plus a
mean-error bound of 1e-2 of max|g_ref|.
"""

import math

import pytest
import torch

import chia_proj_b200 as cp
import oracle

pytestmark = pytest.mark.gpu

REL_MAX, REL_MEAN = 3e-2, 1e-2


def gen(B, H, S, D, dtype, seed, Hkv=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv or H, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv or H, S, D, generator=g).to(dtype)
    do = torch.randn(B, H, S, D, generator=g).to(dtype)
    return q, k, v, do


def oracle_grads(op, q, k, v, do, **kw):
    H, Hkv = q.shape[1], k.shape[1]
    qf, kf, vf = (t.float().clone().requires_grad_() for t in (q, k, v))
    kr = kf.repeat_interleave(H // Hkv, dim=1) if Hkv != H else kf
    vr = vf.repeat_interleave(H // Hkv, dim=1) if Hkv != H else vf
    out = oracle.run_op(op, qf, kr, vr, **kw)
    (out * do.float()).sum().backward()
    return qf.grad, kf.grad, vf.grad


def check_grad(got, ref, what):
    got = got.float().cpu()
    assert torch.isfinite(got).all(), what
    scale = ref.abs().max().item() + 1e-6
    err = (got - ref).abs()
    assert err.max().item() / scale < REL_MAX, f"{what}: rel-max {err.max().item() / scale:.3e}"
    assert err.mean().item() / scale < REL_MEAN, f"{what}: rel-mean {err.mean().item() / scale:.3e}"


def run_case(op, kw, B, H, S, D, dtype, seed, Hkv=None):
    q, k, v, do = gen(B, H, S, D, dtype, seed, Hkv)
    dev = torch.device("cuda", 0)
    qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
    out = cp.OPS[op](qd, kd, vd, **kw)
    out.backward(do.to(dev))
    torch.cuda.synchronize()
    cp.check_device_status(0)
    gq, gk, gv = oracle_grads(op, q, k, v, do, **kw)
    check_grad(qd.grad, gq, f"{op} dq")
    check_grad(kd.grad, gk, f"{op} dk")
    check_grad(vd.grad, gv, f"{op} dv")


CASES = [
    # (op, kwargs, B, H, S, D, dtype)
    ("softcap_gemma2", {}, 1, 2, 300, 128, torch.bfloat16),
    ("softcap_gemma2", dict(cap=50.0, causal=False), 2, 2, 256, 128, torch.bfloat16),
    ("bias_alibi", {}, 1, 3, 400, 128, torch.bfloat16),
    ("bias_alibi", dict(slopes=cp.alibi_slopes_geometric(4)), 1, 4, 512, 128, torch.float16),
    ("temp_perhead", {}, 1, 2, 333, 128, torch.bfloat16),
    ("bias_sliding_window", dict(window=100), 1, 2, 700, 128, torch.bfloat16),
    ("bias_local", dict(window=64), 1, 2, 500, 128, torch.bfloat16),
    ("bias_block_diagonal", dict(block=100), 1, 2, 450, 128, torch.bfloat16),
    ("bias_prefix_lm", dict(prefix=200), 1, 2, 450, 128, torch.bfloat16),
    ("bias_dilated", {}, 1, 2, 512, 128, torch.bfloat16),   # residue-class path
    ("bias_dilated", dict(dilation=3), 1, 2, 301, 128, torch.bfloat16),  # element mask
    ("sigmoid_attn", {}, 1, 2, 300, 128, torch.bfloat16),
    ("sigmoid_attn", dict(causal=False, bias=-math.log(512)), 1, 2, 512, 128, torch.bfloat16),
    ("relu_attn", {}, 1, 2, 300, 128, torch.bfloat16),
    ("relu_attn", dict(causal=False, out_scale=1.0 / 512), 1, 2, 512, 128, torch.bfloat16),
    ("softcap_gemma2", {}, 1, 2, 300, 64, torch.bfloat16),
    ("bias_sliding_window", dict(window=100), 2, 2, 400, 64, torch.float16),
    ("sigmoid_attn", {}, 1, 2, 200, 64, torch.bfloat16),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_gradients_match_autograd_of_the_oracle(cuda, case):
    op, kw, B, H, S, D, dtype = case
    run_case(op, kw, B, H, S, D, dtype, seed=S + D)


@pytest.mark.parametrize("D", [64, 128])
def test_grouped_query_gradients(cuda, D):
    """dK, dV of a K/V head sum the contributions of its query heads."""
    run_case("softcap_gemma2", {}, 1, 8, 300, D, torch.bfloat16, seed=7, Hkv=2)


def test_gradients_are_deterministic_except_dq_order(cuda):
    """dK and dV come from one CTA each (bit-identical across runs); dQ adds
    fp32 partial sums in a run-dependent order (equal to rounding)."""
    q, k, v, do = gen(1, 4, 640, 128, torch.bfloat16, seed=3)
    dev = torch.device("cuda", 0)
    res = []
    for _ in range(2):
        qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
        cp.softcap_gemma2(qd, kd, vd).backward(do.to(dev))
        res.append((qd.grad.clone(), kd.grad.clone(), vd.grad.clone()))
    assert torch.equal(res[0][1], res[1][1]) and torch.equal(res[0][2], res[1][2])
    assert (res[0][0].float() - res[1][0].float()).abs().max().item() < 1e-2
