"""chia_attn_fwd_noalloc (include/chia_attn.h): the entry point that takes no
workspace and allocates nothing, checked against chia_attn_fwd through the C
ABI. The file name makes pytest collect it last; it also passes on its own.
"""

import ctypes

import pytest

from chia_proj_b200 import _native as N

# Tolerance of the operator parity tests, for the check against the oracle.
# Against chia_attn_fwd the comparison is exact: both entry points run the
# same kernel with the same dynamic schedule, and a work unit's result does
# not depend on which CTA runs it.
ATOL = 2e-2


def _params(q, k, v, o, *, norm=N.NORM_SOFTMAX, mod=N.MOD_NONE, left=-1, right=0,
            status=None, workspace=None):
    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.dtype = N.DTYPE_BF16
    B, H, S, D = q.shape
    p.head_dim = D
    p.norm, p.mod = norm, mod
    p.batch, p.heads, p.seqlen_q, p.seqlen_kv = B, H, S, k.shape[2]
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    for field, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", o)):
        getattr(p, field)[:] = t.stride()[:3]
    p.scale = D ** -0.5
    p.softcap, p.sig_bias, p.out_scale = 30.0, 0.0, 1.0
    p.win_left, p.win_right, p.block, p.prefix, p.dilation = left, right, 0, 0, 1
    p.status = status.data_ptr() if status is not None else None
    p.workspace = workspace.data_ptr() if workspace is not None else None
    return p


def _fake_params(**kw):
    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.dtype, p.head_dim, p.norm, p.mod = N.DTYPE_BF16, 128, N.NORM_SOFTMAX, N.MOD_NONE
    p.batch, p.heads, p.seqlen_q, p.seqlen_kv = 1, 1, 128, 128
    p.q = p.k = p.v = p.o = 1 << 20  # never dereferenced: rejected before launch
    p.scale, p.softcap, p.sig_bias, p.out_scale = 0.1, 30.0, 0.0, 1.0
    p.win_left, p.win_right, p.block, p.prefix, p.dilation = -1, 0, 0, 0, 1
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def test_noalloc_rejects_workspace(lib):
    p = _fake_params(workspace=1 << 12)
    assert lib.chia_attn_fwd_noalloc(ctypes.byref(p), None) == 1  # INVALID_ARGUMENT


def test_noalloc_rejects_sizes_beyond_the_scratch_limit(lib):
    # ceil(1 / 256) * batch * heads = 2^30 + 2^15 work units > 2^30
    p = _fake_params(batch=1 << 15, heads=(1 << 15) + 1, seqlen_q=1, seqlen_kv=1)
    assert p.batch * p.heads > N.NOALLOC_MAX_UNITS
    assert lib.chia_attn_fwd_noalloc(ctypes.byref(p), None) == 2  # UNSUPPORTED


def _check_oracle(got, ref):
    import torch
    got = got.float().cpu()
    err = (got - ref).abs().max().item()
    bound = ATOL * max(1.0, ref.abs().max().item())
    assert torch.isfinite(got).all()
    assert err <= bound, f"max |noalloc - oracle| = {err} > {bound}"


@pytest.mark.gpu
def test_noalloc_matches_fwd_on_two_calls(lib, cuda):
    """Two calls in a row through the C ABI: each output is bit-identical to
    chia_attn_fwd's with a caller workspace (the second call also shows that
    the shared scratch was left ready), and the first case also matches the
    fp32 oracle, so a scratch path that is wrong in the same way as the
    other cannot pass."""
    import torch
    import oracle
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    workspace = torch.zeros(N.WORKSPACE_BYTES // 4, dtype=torch.int32, device=cuda)
    gen = torch.Generator(device="cpu").manual_seed(7)
    cases = [
        # (B, H, S, D, norm, window left, window right, oracle check)
        (2, 4, 1000, 128, N.NORM_SOFTMAX, -1, 0, True),    # causal softmax, 2-SM kernel
        (1, 3, 777, 64, N.NORM_SIGMOID, 255, 0, False),    # sliding window, 1-SM kernel
    ]
    for B, H, S, D, norm, left, right, with_oracle in cases:
        qh, kh, vh = (torch.randn(B, H, S, D, generator=gen).to(torch.bfloat16)
                      for _ in range(3))
        q, k, v = qh.to(cuda), kh.to(cuda), vh.to(cuda)
        o_ref = torch.empty_like(q)
        pr = _params(q, k, v, o_ref, norm=norm, left=left, right=right, status=status,
                     workspace=workspace)
        assert lib.chia_attn_fwd(ctypes.byref(pr), stream) == 0
        for call in range(2):
            o_new = torch.full_like(q, float("nan"))
            pn = _params(q, k, v, o_new, norm=norm, left=left, right=right, status=status)
            assert lib.chia_attn_fwd_noalloc(ctypes.byref(pn), stream) == 0
            torch.cuda.synchronize(cuda)
            assert status.item() == 0
            assert torch.equal(o_new, o_ref), f"call {call}: noalloc differs from chia_attn_fwd"
        if with_oracle:
            # plain causal softmax: the dilated operator with dilation 1
            _check_oracle(o_new, oracle.run_op("bias_dilated", qh, kh, vh, dilation=1))
