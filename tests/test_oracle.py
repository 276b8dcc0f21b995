"""The CPU oracle against golden vectors produced by the reference's own code.

``tests/golden/make_golden.py`` executed the reference's ``build_refs``
(``extra_bench.py:32-62``) and ``ref_sigmoid`` (``sigmoid_fix.py:34-40``) on
seeded inputs; the oracle restatement must reproduce them, and its
generalised parameters must reduce to the reference at their defaults.
"""

import math

import pytest
import torch

import oracle
from oracle import eager


@pytest.mark.parametrize("op", sorted(oracle.OPS))
def test_oracle_matches_reference_golden(golden, op):
    out = oracle.run_op(op, golden["q"], golden["k"], golden["v"])
    ref = golden["outputs"][op]
    assert out.shape == ref.shape
    torch.testing.assert_close(out, ref, rtol=0, atol=1e-6)


def test_oracle_sigmoid_is_the_corrected_reference(golden):
    out = oracle.run_op("sigmoid_attn", golden["q"], golden["k"], golden["v"])
    torch.testing.assert_close(out, golden["outputs"]["sigmoid_fix.ref_sigmoid"], rtol=0,
                               atol=1e-6)


def _inputs(B=1, H=3, S=200, D=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, S, D, generator=g) for _ in range(3)]


def test_explicit_defaults_equal_reference_defaults():
    q, k, v = _inputs()
    H = q.shape[1]
    torch.testing.assert_close(eager.bias_alibi(q, k, v, slopes=torch.arange(1, H + 1.0)),
                               eager.bias_alibi(q, k, v), rtol=0, atol=0)
    torch.testing.assert_close(eager.temp_perhead(q, k, v, temps=0.5 + torch.arange(H) / H),
                               eager.temp_perhead(q, k, v), rtol=0, atol=0)
    torch.testing.assert_close(eager.softcap_gemma2(q, k, v, cap=30.0, causal=True),
                               eager.softcap_gemma2(q, k, v), rtol=0, atol=0)


def test_generalised_parameters_behave():
    q, k, v = _inputs(S=300)
    S = q.shape[2]
    # huge cap -> plain causal softmax
    plain = eager._eval(q, k, v, maskfn=eager.reference_masks()["causal"])
    torch.testing.assert_close(eager.softcap_gemma2(q, k, v, cap=1e7), plain, rtol=1e-4,
                               atol=1e-5)
    # sigmoid bias: sigmoid(s + b) computed directly
    b = -math.log(S)
    s = (q @ k.transpose(-2, -1)) / math.sqrt(q.shape[-1])
    direct = torch.sigmoid(s + b) @ v
    torch.testing.assert_close(eager.sigmoid_attn(q, k, v, causal=False, bias=b), direct,
                               rtol=1e-5, atol=1e-5)
    # relu out_scale is linear
    torch.testing.assert_close(eager.relu_attn(q, k, v, causal=False, out_scale=1.0 / S),
                               eager.relu_attn(q, k, v, causal=False) / S, rtol=1e-6, atol=1e-7)
    # non-causal block-diagonal: each block is independent full attention
    bd = eager.bias_block_diagonal(q, k, v, block=100, causal=False)
    for b0 in range(0, S, 100):
        sl = slice(b0, min(S, b0 + 100))
        blk = eager._eval(q[:, :, sl], k[:, :, sl], v[:, :, sl],
                          maskfn=eager.reference_masks()["full"])
        torch.testing.assert_close(bd[:, :, sl], blk, rtol=1e-5, atol=1e-6)


def test_oracle_row_blocking_is_invisible():
    q, k, v = _inputs(S=130)
    a = eager._eval(q, k, v, maskfn=eager.reference_masks()["causal"], row_block=7)
    b = eager._eval(q, k, v, maskfn=eager.reference_masks()["causal"], row_block=1024)
    torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)


def test_varlen_oracle_is_the_operator_per_sequence():
    """Packed sequences: each sequence's output is the operator on that
    sequence alone, so tokens of other sequences do not affect it."""
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 50, 16, generator=g) for _ in range(3))
    cu = [0, 20, 20, 50]
    out = oracle.run_varlen("softcap_gemma2", q, k, v, cu)
    alone = oracle.run_op("softcap_gemma2", q[:, :, 20:], k[:, :, 20:], v[:, :, 20:])
    assert torch.equal(out[:, :, 20:], alone)
    k2 = k.clone()
    k2[:, :, :20] += 5.0
    assert torch.equal(oracle.run_varlen("softcap_gemma2", q, k2, v, cu)[:, :, 20:], out[:, :, 20:])
