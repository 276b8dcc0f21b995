"""GPU parity: the sm_100a kernel against the fp32 CPU oracle.

Bar: max-abs <= 2e-2 and mean-abs <= 2e-3 against the
fp32 eager reference for bf16/fp16 inputs. The reference's own acceptance
gate, ``max|r-o| / max|r| < 3e-2`` (``synth10.py:15,182-184``), is checked
as well, because outputs of some variants (ReLU/S, sigmoid - log S) are so
small that absolute bounds alone would pass a wrong kernel.

The absolute bounds assume O(1) outputs, which holds for every softmax
variant and for the benchmark's sigmoid (bias -log S) and ReLU (scale 1/S).
With the reference's default parameters sigmoid and ReLU are unnormalised
and outputs grow like sqrt(S) (|o| ~ 30 at S=256): rounding the output to
bf16 alone then costs |o| * 2^-9. The bounds are therefore multiplied by
max(1, max|ref|) -- a no-op for O(1) outputs. The error there is the same
bf16 rounding of P that the reference's own ``p.to(DT)`` performs.
"""

import math

import pytest
import torch

import chia_proj_b200 as cp
import oracle

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS, REL_MAX = 2e-2, 2e-3, 3e-2


def gen(B, H, S, D, dtype, seed=0, scale=1.0, Skv=None):
    g = torch.Generator().manual_seed(seed)
    shp = lambda s: (B, H, s, D)
    q = (torch.randn(*shp(S), generator=g) * scale).to(dtype)
    k = (torch.randn(*shp(Skv or S), generator=g) * scale).to(dtype)
    v = (torch.randn(*shp(Skv or S), generator=g) * scale).to(dtype)
    return q, k, v


def check(out, ref, what=""):
    out = out.float().cpu()
    assert out.shape == ref.shape, what
    assert torch.isfinite(out).all(), what
    err = (out - ref).abs()
    rmax = ref.abs().max().item()
    rel = err.max().item() / (rmax + 1e-6)
    tol_max = MAX_ABS * max(1.0, rmax)
    tol_mean = MEAN_ABS * max(1.0, rmax)
    assert err.max().item() <= tol_max, f"{what}: max-abs {err.max().item():.3e} > {tol_max:.3e}"
    assert err.mean().item() <= tol_mean, f"{what}: mean-abs {err.mean().item():.3e}"
    assert rel < REL_MAX, f"{what}: rel-max {rel:.3e}"


def run(op, q, k, v, **kw):
    dev = torch.device("cuda", 0)
    out = cp.OPS[op](q.to(dev), k.to(dev), v.to(dev), **kw)
    torch.cuda.synchronize()
    return out


@pytest.fixture(autouse=True)
def _status_clean(cuda):
    yield
    cp.check_device_status(0)


# ------------------------------------------------------------------ golden
@pytest.mark.parametrize("op", sorted(cp.OPS))
def test_golden_reference_vectors(cuda, golden, op):
    """Outputs the reference's own eager code produced (tests/golden/)."""
    out = run(op, golden["q"], golden["k"], golden["v"])
    check(out, golden["outputs"][op], op)


# ------------------------------------------------------- reference defaults
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [1, 100, 129, 384, 1000])
@pytest.mark.parametrize("op", sorted(cp.OPS))
def test_reference_defaults(cuda, op, S, D, dtype):
    q, k, v = gen(1, 2, S, D, dtype, seed=S + D)
    ref = oracle.run_op(op, q, k, v)
    check(run(op, q, k, v), ref, f"{op} S={S} D={D} {dtype}")


@pytest.mark.parametrize("op", sorted(cp.OPS))
def test_small_input_scale(cuda, op):
    """The reference gate's second input scale, 0.01 (synth10.py:175-177)."""
    q, k, v = gen(2, 2, 300, 128, torch.bfloat16, seed=7, scale=0.01)
    ref = oracle.run_op(op, q, k, v)
    out = run(op, q, k, v).float().cpu()
    err = (out - ref).abs().max().item()
    assert err / (ref.abs().max().item() + 1e-6) < REL_MAX, op


# ---------------------------------------------------- benchmark parameters
def _tau(H, seed=0):
    g = torch.Generator().manual_seed(seed)
    return 0.5 + 1.5 * torch.rand(H, generator=g)


BASELINE_CASES = [
    # (op, kwargs, oracle kwargs, B, H, S, D, dtype)
    ("softcap_gemma2", dict(cap=50.0, causal=False), dict(cap=50.0, causal=False),
     1, 2, 512, 64, torch.bfloat16),
    ("bias_sliding_window", dict(window=256), dict(window=256), 1, 2, 2048, 64, torch.bfloat16),
    ("bias_alibi", dict(slopes=cp.alibi_slopes_geometric(4)),
     dict(slopes=cp.alibi_slopes_geometric(4)), 1, 4, 1024, 128, torch.float16),
    ("temp_perhead", dict(temps=1.0 / _tau(4)), dict(temps=1.0 / _tau(4)),
     1, 4, 1024, 128, torch.float16),
    ("bias_prefix_lm", dict(prefix=1024), dict(prefix=1024), 1, 2, 1500, 128, torch.bfloat16),
    ("bias_block_diagonal", dict(block=256), dict(block=256), 1, 2, 1024, 128, torch.bfloat16),
    ("bias_block_diagonal", dict(block=256, causal=False), dict(block=256, causal=False),
     1, 2, 1024, 128, torch.bfloat16),
    ("bias_dilated", dict(dilation=4), dict(dilation=4), 1, 2, 1024, 128, torch.bfloat16),
    ("bias_dilated", dict(dilation=4), dict(dilation=4), 1, 2, 1023, 128, torch.bfloat16),
    ("bias_dilated", dict(dilation=3), dict(dilation=3), 2, 1, 999, 64, torch.bfloat16),
    ("sigmoid_attn", dict(causal=False, bias=-math.log(2048)),
     dict(causal=False, bias=-math.log(2048)), 1, 2, 2048, 128, torch.bfloat16),
    ("relu_attn", dict(causal=False, out_scale=1.0 / 2048), dict(causal=False, out_scale=1.0 / 2048),
     1, 2, 2048, 128, torch.bfloat16),
    ("bias_local", dict(window=100), dict(window=100), 1, 2, 700, 64, torch.bfloat16),
    ("bias_block_diagonal", dict(block=100), dict(block=100), 1, 2, 700, 64, torch.float16),
    ("bias_prefix_lm", dict(prefix=200), dict(prefix=200), 1, 2, 700, 64, torch.bfloat16),
    ("bias_sliding_window", dict(window=1), dict(window=1), 1, 2, 300, 64, torch.bfloat16),
]


@pytest.mark.parametrize("case", BASELINE_CASES,
                         ids=[f"{c[0]}-{i}" for i, c in enumerate(BASELINE_CASES)])
def test_benchmark_parameters(cuda, case):
    op, kw, okw, B, H, S, D, dtype = case
    q, k, v = gen(B, H, S, D, dtype, seed=S)
    ref = oracle.run_op(op, q, k, v, **okw)
    check(run(op, q, k, v, **kw), ref, f"{op} {kw}")


# ------------------------------------------------------------------ layouts
def test_strided_inputs(cuda):
    """[B, S, H, D] storage viewed as [B, H, S, D] (non-contiguous, TMA strides)."""
    B, H, S, D = 2, 3, 333, 128
    g = torch.Generator().manual_seed(3)
    base = [torch.randn(B, S, H, D, generator=g).to(torch.bfloat16) for _ in range(3)]
    q, k, v = (t.transpose(1, 2) for t in base)
    ref = oracle.run_op("softcap_gemma2", q, k, v)
    dev = torch.device("cuda", 0)
    qd, kd, vd = (t.to(dev).transpose(1, 2) for t in base)
    assert not qd.is_contiguous()
    check(cp.softcap_gemma2(qd, kd, vd), ref, "strided")


def test_fp32_inputs_accepted(cuda):
    """Config-1 shape in fp32: fp16 operands (the mantissa of a TF32 MMA) with
    fp32 accumulation, an order of magnitude closer to the fp32 reference than
    bf16 operands, which remain available through ``compute_dtype``."""
    q, k, v = gen(1, 8, 512, 64, torch.float32, seed=1)
    ref = oracle.run_op("softcap_gemma2", q, k, v, cap=50.0, causal=False)
    out = run("softcap_gemma2", q, k, v, cap=50.0, causal=False)
    assert out.dtype == torch.float32
    check(out, ref, "fp32 config 1")
    dev = torch.device("cuda", 0)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    kw = dict(mod="softcap", softcap=50.0, mask=cp.FULL)
    o16 = cp.attention(qd, kd, vd, **kw).cpu()
    obf = cp.attention(qd, kd, vd, compute_dtype=torch.bfloat16, **kw).cpu()
    e16, ebf = (o16 - ref).abs(), (obf - ref).abs()
    assert torch.equal(o16, out.cpu())
    assert e16.max() < 2e-3 and e16.mean() < 2e-4, (e16.max(), e16.mean())
    assert e16.max() < 0.25 * ebf.max() and e16.mean() < 0.25 * ebf.mean()


def test_fp32_inputs_outside_fp16_range_use_bf16(cuda):
    """Inputs (or ReLU scores) that fp16 cannot hold fall back to bf16 operands."""
    q, k, v = gen(1, 2, 256, 64, torch.float32, seed=3)
    dev = torch.device("cuda", 0)
    big = v.clone()
    big[0, 0, 0, 0] = 1.0e5  # row 0 sees key 0 alone: its output is this value
    ref = oracle.run_op("bias_dilated", q, k, big, dilation=1)
    out = cp.attention(q.to(dev), k.to(dev), big.to(dev))
    assert torch.isfinite(out).all()
    forced = cp.attention(q.to(dev), k.to(dev), big.to(dev), compute_dtype=torch.bfloat16)
    assert torch.equal(out, forced)
    # ReLU: P = relu(s * scale) reaches 8 * 8 * 64 / 8 = 512 here but 5e5 with
    # 100-fold inputs, which fp16 cannot hold
    q2, k2 = q * 100.0, k * 100.0
    o_auto = cp.attention(q2.to(dev), k2.to(dev), v.to(dev), norm="relu", mask=cp.FULL)
    o_bf = cp.attention(q2.to(dev), k2.to(dev), v.to(dev), norm="relu", mask=cp.FULL,
                        compute_dtype=torch.bfloat16)
    assert torch.equal(o_auto, o_bf)
    with pytest.raises(ValueError):
        cp.attention(q2.to(dev).half(), k2.to(dev).half(), v.to(dev).half(),
                     compute_dtype=torch.bfloat16)
    check(out, ref, "fp32, element out of fp16 range")


def _eager_dt(op, q, k, v):
    """The reference's eager operator evaluated in the inputs' 16-bit type,
    as its own benchmark harness runs it (``extra_bench.py:38-45``): scores
    rounded to DT, the normaliser in fp32, ``p.to(DT) @ v``. Sigmoid and ReLU
    at the reference's defaults (causal, no bias, no output scale)."""
    S, D = q.shape[-2], q.shape[-1]
    s = (q @ k.transpose(-2, -1)) * (1.0 / math.sqrt(D))
    i = torch.arange(S).view(-1, 1)
    j = torch.arange(S).view(1, -1)
    ok = (j <= i).float()
    p = torch.sigmoid(s.float()) * ok if op == "sigmoid_attn" else torch.relu(s.float()) * ok
    return (p.to(q.dtype) @ v).float()


@pytest.mark.parametrize("op", ["sigmoid_attn", "relu_attn"])
def test_unnormalised_defaults_no_worse_than_bf16_eager(cuda, op):
    """At the reference's default parameters sigmoid and ReLU outputs grow like
    sqrt(S), so ``check`` scales its absolute bounds by max|ref|. This measures
    what that allowance is for: the reference's own eager computation in bf16
    misses its fp32 result by at least as much as the kernel does."""
    q, k, v = gen(1, 4, 512, 128, torch.bfloat16, seed=21)
    ref = oracle.run_op(op, q, k, v)
    out = run(op, q, k, v).float().cpu()
    eager = _eager_dt(op, q, k, v)
    e_k, e_e = (out - ref).abs(), (eager - ref).abs()
    assert e_k.max() <= 1.1 * e_e.max(), (e_k.max(), e_e.max())
    assert e_k.mean() <= 1.1 * e_e.mean(), (e_k.mean(), e_e.mean())


def test_preallocated_output(cuda):
    q, k, v = gen(1, 2, 256, 64, torch.bfloat16, seed=2)
    dev = torch.device("cuda", 0)
    out = torch.full((1, 2, 256, 64), float("nan"), dtype=torch.bfloat16, device=dev)
    r = cp.attention(q.to(dev), k.to(dev), v.to(dev), out=out)
    assert r.data_ptr() == out.data_ptr()
    check(out, oracle.run_op("bias_dilated", q, k, v, dilation=1), "out=")


# ------------------------------------------- full-size, size-independent checks
def test_linearity_in_v_is_exact(cuda):
    q, k, v = gen(1, 4, 2048, 128, torch.bfloat16, seed=11)
    dev = torch.device("cuda", 0)
    q, k, v = q.to(dev), k.to(dev), v.to(dev)
    for op in cp.OPS:
        a = cp.OPS[op](q, k, v)
        b = cp.OPS[op](q, k, v * 2)
        assert torch.equal(a * 2, b), op


@pytest.mark.parametrize("op,kw", [
    ("bias_sliding_window", {}), ("bias_block_diagonal", dict(block=256)),
    ("bias_prefix_lm", dict(prefix=1024)), ("bias_dilated", {}), ("softcap_gemma2", {}),
    ("bias_local", {}),
    # the causal kinds the headline suite times
    ("bias_alibi", dict(slopes=cp.alibi_slopes_geometric(16))),
    ("temp_perhead", dict(temps=1.0 / _tau(16))),
    ("softcap_gemma2", dict(cap=50.0)),
    ("sigmoid_attn", {}),
    ("relu_attn", dict(out_scale=1.0 / 4096)),
])
def test_invisible_keys_do_not_matter_at_headline_shape(cuda, op, kw):
    """B4 H16 S4096 D128: perturbing keys/values a mask hides leaves the output
    bit-identical; two sampled heads also match the oracle."""
    B, H, S, D = 4, 16, 4096, 128
    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in gen(B, H, S, D, torch.bfloat16, seed=5))
    out = cp.OPS[op](q, k, v, **kw)
    # perturb keys/values of query rows [3000, 3100) that are invisible to all of them
    mask = cp.op_config(op, **kw)
    i = torch.arange(3000, 3100).view(-1, 1)
    j = torch.arange(S).view(1, -1)
    vis = torch.zeros(100, S, dtype=torch.bool)
    band = torch.ones_like(vis)
    if mask.left >= 0:
        band &= (i - j) <= mask.left
    if mask.right >= 0:
        band &= (j - i) <= mask.right
    if mask.block > 0:
        band &= (i // mask.block) == (j // mask.block)
    band &= ((i - j) % mask.dilation) == 0
    vis = band | (j < mask.prefix)
    hidden = (~vis.any(0)).nonzero().flatten().to(dev)
    k2, v2 = k.clone(), v.clone()
    k2[:, :, hidden] = torch.randn_like(k2[:, :, hidden]) * 3
    v2[:, :, hidden] = torch.randn_like(v2[:, :, hidden]) * 3
    out2 = cp.OPS[op](q, k2, v2, **kw)
    assert torch.equal(out[:, :, 3000:3100], out2[:, :, 3000:3100])
    for (b, h) in ((0, 0), (3, 15)):
        # per-head parameters follow the sliced head
        okw = {n: (x[h:h + 1] if n in ("slopes", "temps") else x) for n, x in kw.items()}
        ref = oracle.run_op(op, q[b:b + 1, h:h + 1].cpu(), k[b:b + 1, h:h + 1].cpu(),
                            v[b:b + 1, h:h + 1].cpu(), **okw)
        check(out[b:b + 1, h:h + 1], ref, f"{op} head ({b},{h})")


@pytest.mark.parametrize("op", ["bias_alibi", "temp_perhead"])
def test_config3_at_its_own_shape(cuda, op):
    """BASELINE config 3 exactly as the bench times it: B8 H32 S4096 D128 fp16,
    causal; ALiBi slopes 2^(-8(h+1)/H), temperatures 1/tau_h with
    tau_h ~ U[0.5, 2] from seed 0. Three sampled heads against the oracle,
    among them the last head (smallest slope, 2^-8)."""
    B, H, S, D = 8, 32, 4096, 128
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=dev).to(torch.float16)
               for _ in range(3))
    if op == "bias_alibi":
        kw = dict(slopes=cp.alibi_slopes_geometric(H))
    else:
        kw = dict(temps=1.0 / _tau(H))
    out = cp.OPS[op](q, k, v, **kw)
    torch.cuda.synchronize()
    for (b, h) in ((0, 0), (3, 17), (7, 31)):
        sl = lambda x: x[b:b + 1, h:h + 1].cpu()
        okw = dict(slopes=kw["slopes"][h:h + 1]) if op == "bias_alibi" else \
            dict(temps=kw["temps"][h:h + 1])
        ref = oracle.run_op(op, sl(q), sl(k), sl(v), **okw)
        check(out[b:b + 1, h:h + 1], ref, f"{op} config 3 head ({b},{h})")


def test_config2_every_head(cuda):
    """BASELINE config 2 in full: causal sliding window 256, B4 H16 S2048
    D64 bf16, all 64 heads against the oracle."""
    q, k, v = gen(4, 16, 2048, 64, torch.bfloat16, seed=2)
    ref = oracle.run_op("bias_sliding_window", q, k, v, window=256)
    check(run("bias_sliding_window", q, k, v, window=256), ref, "config 2")


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("op,kw", [("softcap_gemma2", {}), ("bias_sliding_window", {}),
                                   ("bias_alibi", {}), ("bias_dilated", {}),
                                   ("bias_prefix_lm", dict(prefix=300)),
                                   ("softcap_gemma2", dict(cap=50.0, causal=False))])
def test_log_sum_exp_output(cuda, op, kw, D):
    """The per-row log-sum-exp the forward writes for the backward pass,
    against the oracle's, on a ragged length."""
    q, k, v = gen(2, 3, 1000, D, torch.bfloat16, seed=D + 5)
    ref_o, ref_lse = oracle.run_op_lse(op, q, k, v, **kw)
    dev = torch.device("cuda", 0)
    mask = cp.op_config(op, **kw)
    mod = {"softcap_gemma2": "softcap", "bias_alibi": "alibi"}.get(op, "none")
    extra = dict(softcap=kw.get("cap", 30.0)) if mod == "softcap" else {}
    o, lse = cp.attention(q.to(dev), k.to(dev), v.to(dev), mod=mod, mask=mask,
                          return_lse=True, **extra)
    torch.cuda.synchronize()
    check(o, ref_o, f"{op} D={D}")
    err = (lse.cpu() - ref_lse).abs().max().item()
    assert err < 1e-3, f"{op} D={D}: lse max error {err}"


def test_log_sum_exp_of_rows_without_keys(cuda):
    """Rows that see no key (S_q > S_kv with a window) get -inf."""
    dev = torch.device("cuda", 0)
    q, _, _ = gen(1, 2, 600, 128, torch.bfloat16, seed=83)
    _, k, v = gen(1, 2, 128, 128, torch.bfloat16, seed=84)
    o, lse = cp.attention(q.to(dev), k.to(dev), v.to(dev), mask=cp.Mask(left=63, right=0),
                          return_lse=True)
    torch.cuda.synchronize()
    lse = lse.cpu()
    assert torch.isinf(lse[:, :, 191:]).all() and (lse[:, :, 191:] < 0).all()
    assert torch.isfinite(lse[:, :, :191]).all()


@pytest.mark.parametrize("op", ["sigmoid_attn", "relu_attn"])
def test_config5_heads_match_oracle(cuda, op):
    """Config 5 shape per head (S=8192, D=128, non-causal): sampled heads."""
    S = 8192
    kw = dict(causal=False, bias=-math.log(S)) if op == "sigmoid_attn" else \
        dict(causal=False, out_scale=1.0 / S)
    q, k, v = gen(1, 3, S, 128, torch.bfloat16, seed=9)
    out = run(op, q, k, v, **kw)
    ref = oracle.run_op(op, q[:, :2], k[:, :2], v[:, :2], **kw)
    check(out[:, :2], ref, op)


def test_repeat_calls_are_deterministic(cuda):
    q, k, v = gen(2, 4, 1000, 128, torch.bfloat16, seed=4)
    dev = torch.device("cuda", 0)
    q, k, v = q.to(dev), k.to(dev), v.to(dev)
    a = cp.bias_alibi(q, k, v, slopes=cp.alibi_slopes_geometric(4))
    for _ in range(3):
        assert torch.equal(a, cp.bias_alibi(q, k, v, slopes=cp.alibi_slopes_geometric(4)))


@pytest.mark.parametrize("op", ["softcap_gemma2", "bias_sliding_window", "sigmoid_attn"])
def test_static_and_dynamic_schedules_agree(cuda, op):
    """Both work schedules run the same units; outputs are bit-identical, and
    the dynamic scheduler leaves its workspace zeroed after every call."""
    from chia_proj_b200 import ops
    B, H, S, D = 3, 5, 1500, 128   # 6 query blocks x 15 heads = 90 units < 148 SMs
    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in gen(B, H, S, D, torch.bfloat16, seed=21))
    mask = cp.op_config(op)
    norm = "sigmoid" if op == "sigmoid_attn" else "softmax"
    mod = "softcap" if op == "softcap_gemma2" else "none"
    a = cp.attention(q, k, v, mask=mask, norm=norm, mod=mod, schedule="dynamic")
    b = cp.attention(q, k, v, mask=mask, norm=norm, mod=mod, schedule="static")
    assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert int(ops._workspace(dev).abs().sum()) == 0
    # many more units than SMs
    q, k, v = (t.to(dev) for t in gen(8, 32, 1024, 64, torch.bfloat16, seed=22))
    a = cp.attention(q, k, v, mask=mask, norm=norm, mod=mod, schedule="dynamic")
    b = cp.attention(q, k, v, mask=mask, norm=norm, mod=mod, schedule="static")
    assert torch.equal(a, b)
    torch.cuda.synchronize()
    assert int(ops._workspace(dev).abs().sum()) == 0


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("op,kw", [("bias_alibi", {}), ("softcap_gemma2", dict(cap=1000.0))])
def test_running_max_rises_every_tile(cuda, op, D, kw):
    """Scores grow along the keys by ~12 (log2 units) per 128-key tile, so the
    running row maximum rises on every tile and O is rescaled on every tile
    while earlier P.V products may still be in flight on the tensor core."""
    B, H, S = 1, 4, 2048
    g = torch.Generator().manual_seed(31)
    q = torch.ones(B, H, S, D)
    # score(i, j) = sqrt(D) * k_j: 8.7 nats = 12.5 log2 units more per 128 keys
    ramp = torch.arange(S, dtype=torch.float32).view(1, 1, S, 1) * (8.7 / (128 * D ** 0.5))
    k = ramp + 0.1 * torch.randn(B, H, S, D, generator=g)
    v = torch.randn(B, H, S, D, generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    if op == "bias_alibi":
        kw = dict(slopes=torch.zeros(H))
    out = run(op, q, k, v, **kw)
    check(out, oracle.run_op(op, q, k, v, **kw), op)
    for _ in range(3):
        assert torch.equal(out, run(op, q, k, v, **kw))


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [False, True])
def test_sigmoid_logits_whose_exponential_overflows(cuda, D, dtype, causal):
    """Scores of spread 20 with bias -60: t = -(s - 60) log2(e) runs from
    about 0 to 200, so 2^t overflows to inf for roughly a tenth of the pairs
    (sigmoid there is below 1e-38) while the rest span the whole curve. Each
    such P must come out 0, every other one as in the oracle."""
    q, k, v = gen(1, 4, 640, D, dtype, seed=43)
    q, k = ((x.float() * math.sqrt(20.0)).to(dtype) for x in (q, k))  # s ~ N(0, 20^2)
    kw = dict(causal=causal, bias=-60.0)
    s = (q.float() @ k.float().transpose(-2, -1)) / math.sqrt(D)
    t = -(s - 60.0) * math.log2(math.e)
    assert (t >= 128).float().mean() > 0.02 and (t < 40).float().mean() > 0.02
    check(run("sigmoid_attn", q, k, v, **kw), oracle.run_op("sigmoid_attn", q, k, v, **kw),
          f"sigmoid overflow D={D}")


@pytest.mark.parametrize("S", [1024, 1000])
@pytest.mark.parametrize("op,kw", [("softcap_gemma2", dict(cap=50.0, causal=False)),
                                   ("sigmoid_attn", dict(causal=False, bias=-2.0)),
                                   ("relu_attn", dict(causal=False, out_scale=1e-3))])
def test_non_causal_with_and_without_mask_code(cuda, op, kw, S):
    """Non-causal masks with S a multiple of 128 run the kernel built without
    element-wise mask code; S = 1000 leaves a ragged last key tile that must
    still be masked. Both against the oracle."""
    q, k, v = gen(2, 2, S, 128, torch.bfloat16, seed=41)
    check(run(op, q, k, v, **kw), oracle.run_op(op, q, k, v, **kw), f"{op} S={S}")


# ------------------------------------------------------ grouped-query K/V
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("op,kw", [("softcap_gemma2", {}), ("bias_sliding_window", {}),
                                   ("bias_alibi", {}), ("sigmoid_attn", {}),
                                   ("relu_attn", dict(causal=False, out_scale=1e-3))])
def test_grouped_query_heads(cuda, op, kw, D):
    """K/V with fewer heads than Q (8 query heads, 2 K/V heads): the oracle on
    K/V repeated per query head, and bit-identical to passing those repeated
    K/V to the kernel."""
    B, H, Hkv, S = 1, 8, 2, 700
    q, _, _ = gen(B, H, S, D, torch.bfloat16, seed=51)
    _, k, v = gen(B, Hkv, S, D, torch.bfloat16, seed=52)
    kr, vr = (x.repeat_interleave(H // Hkv, dim=1) for x in (k, v))
    out = run(op, q, k, v, **kw)
    check(out, oracle.run_op(op, q, kr, vr, **kw), f"{op} D={D}")
    assert torch.equal(out, run(op, q, kr, vr, **kw))


# ------------------------------------------------ packed variable-length sequences
VARLEN_OFFSETS = [0, 100, 400, 417, 1017, 1017, 1272]  # includes an empty sequence


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("op,kw", [("softcap_gemma2", {}), ("bias_sliding_window", {}),
                                   ("bias_local", dict(window=64)), ("bias_alibi", {}),
                                   ("temp_perhead", {}),
                                   ("sigmoid_attn", dict(causal=False)),
                                   ("relu_attn", dict(out_scale=1e-2))])
def test_packed_sequences_match_per_sequence_oracle(cuda, op, kw, D):
    """cu_seqlens: every sequence attends only to itself, equal to the
    reference operator applied to each sequence alone."""
    S = VARLEN_OFFSETS[-1]
    q, k, v = gen(1, 3, S, D, torch.bfloat16, seed=61)
    out = run(op, q, k, v, cu_seqlens=VARLEN_OFFSETS, **kw)
    check(out, oracle.run_varlen(op, q, k, v, VARLEN_OFFSETS, **kw), f"{op} D={D}")


def test_packed_sequences_device_offsets_and_isolation(cuda):
    """int32 offsets already on the device give the same result, and keys of
    other sequences do not change a sequence's output (bit-exact)."""
    S = VARLEN_OFFSETS[-1]
    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in gen(1, 2, S, 128, torch.bfloat16, seed=62))
    cu = torch.tensor(VARLEN_OFFSETS, dtype=torch.int32, device=dev)
    a = cp.softcap_gemma2(q, k, v, cu_seqlens=VARLEN_OFFSETS)
    assert torch.equal(a, cp.softcap_gemma2(q, k, v, cu_seqlens=cu))
    k2, v2 = k.clone(), v.clone()
    k2[:, :, :400] = torch.randn_like(k2[:, :, :400]) * 3
    v2[:, :, :400] = torch.randn_like(v2[:, :, :400]) * 3
    b = cp.softcap_gemma2(q, k2, v2, cu_seqlens=cu)
    assert torch.equal(a[:, :, 400:], b[:, :, 400:])


# ------------------------------------------------ decode-shaped calls (S_q < S_kv)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Sq,Skv", [(1, 1000), (16, 1024), (200, 1000)])
@pytest.mark.parametrize("norm", ["softmax", "sigmoid", "relu"])
def test_decode_shaped_bottom_right_causal(cuda, norm, Sq, Skv, D):
    """Few queries over a long key sequence, causal aligned at the end (query
    i sits at position Skv - Sq + i: Mask(left=-1, right=Skv-Sq)), with
    grouped K/V heads; against the oracle's generic evaluator."""
    from oracle import eager
    off = Skv - Sq
    H, Hkv = 4, 2
    q, _, _ = gen(2, H, Sq, D, torch.bfloat16, seed=71)
    _, k, v = gen(2, Hkv, Skv, D, torch.bfloat16, seed=72)
    kw = dict(sig_bias=-math.log(Skv)) if norm == "sigmoid" else \
        dict(out_scale=1.0 / Skv) if norm == "relu" else {}
    dev = torch.device("cuda", 0)
    out = cp.attention(q.to(dev), k.to(dev), v.to(dev), norm=norm,
                       mask=cp.Mask(left=-1, right=off), **kw)
    kr, vr = (x.repeat_interleave(H // Hkv, dim=1) for x in (k, v))
    if norm == "sigmoid":
        ref = eager._eval(q, kr, vr, maskfn=lambda i, j: j <= i + off, norm="sigmoid",
                          mod=lambda s, h, i, j: s + kw["sig_bias"])
    else:
        ref = eager._eval(q, kr, vr, maskfn=lambda i, j: j <= i + off, norm=norm)
        if norm == "relu":
            ref = ref * kw["out_scale"]
    check(out, ref, f"{norm} Sq={Sq} Skv={Skv}")


# ------------------------------------------- work units whose rows see no key
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("norm", ["softmax", "sigmoid"])
def test_keyless_units_write_zeros(cuda, norm, D):
    """Query rows past the last visible key (S_q > S_kv, a window of 64):
    rows 191.. see no key, so whole work units have no key tile. Their
    output is zero -- written over a pre-filled buffer -- and the units in
    between keep the pipeline's tile and buffer order intact."""
    from oracle import eager
    Sq, Skv, W = 1024, 128, 64
    q, _, _ = gen(2, 3, Sq, D, torch.bfloat16, seed=81)
    _, k, v = gen(2, 3, Skv, D, torch.bfloat16, seed=82)
    kw = dict(sig_bias=-math.log(Skv)) if norm == "sigmoid" else {}
    dev = torch.device("cuda", 0)
    out = torch.full((2, 3, Sq, D), 7.0, dtype=torch.bfloat16, device=dev)
    for schedule in ("dynamic", "static"):
        cp.attention(q.to(dev), k.to(dev), v.to(dev), norm=norm, out=out,
                     mask=cp.Mask(left=W - 1, right=0), schedule=schedule, **kw)
        torch.cuda.synchronize()
        maskfn = lambda i, j: (j <= i) & (j > i - W)
        if norm == "sigmoid":
            ref = eager._eval(q, k, v, maskfn=maskfn, norm="sigmoid",
                              mod=lambda s, h, i, j: s + kw["sig_bias"])
        else:
            ref = torch.nan_to_num(eager._eval(q, k, v, maskfn=maskfn, norm=norm), nan=0.0)
        got = out.float().cpu()
        assert (got[:, :, Skv + W - 1:] == 0).all(), "keyless rows must be zero"
        check(out, ref, f"{norm} D={D} {schedule}")
        out.fill_(7.0)


# ------------------------------------------ two streams, dynamic schedule
def test_concurrent_streams_do_not_share_a_scheduler(cuda):
    """Launches on two streams of one device may overlap on the GPU; each
    stream has its own scheduler workspace, so every unit still runs exactly
    once: outputs equal the static schedule's, bit for bit, and every
    workspace is left zeroed."""
    from chia_proj_b200 import ops
    dev = torch.device("cuda", 0)
    inputs = [tuple(t.to(dev) for t in gen(4, 16, 2048, D, torch.bfloat16, seed=90 + D))
              for D in (128, 64)]
    want = [cp.softcap_gemma2(*x, cap=50.0) for x in inputs]
    want_static = [cp.attention(*x, mod="softcap", softcap=50.0, schedule="static")
                   for x in inputs]
    for a, b in zip(want, want_static):
        assert torch.equal(a, b)
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    got = [[], []]
    for rep in range(6):
        for si, st in enumerate(streams):
            with torch.cuda.stream(st):
                x = inputs[(rep + si) % 2]
                for t in x:
                    t.record_stream(st)
                got[si].append(((rep + si) % 2, cp.softcap_gemma2(*x, cap=50.0)))
    torch.cuda.synchronize()
    for lst in got:
        for which, o in lst:
            assert torch.equal(o, want[which])
    for st in streams:
        assert int(ops._workspace(dev, st.cuda_stream).abs().sum()) == 0


# ------------------------------------------------ a bounded wait that runs out
@pytest.mark.parametrize("D", [128, 64])
def test_wait_that_runs_out_is_reported_and_the_device_recovers(cuda, D):
    """With a wait limit of a few nanoseconds the first wait that is not met
    at once runs out: the kernel sets CHIA_ERR_DEVICE_TIMEOUT in the status
    word, drains its own copies and MMAs, frees its tensor memory and
    returns (no trap, no hang). check_device_status() raises it, and the next
    call with the default limit on the same device is correct and leaves the
    scheduler workspace zeroed."""
    from chia_proj_b200 import ops
    dev = torch.device("cuda", 0)
    q, k, v = gen(2, 4, 2048, D, torch.bfloat16, seed=95)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    cp.check_device_status(0)
    code = 0
    for _ in range(3):   # a wait that happens to be met at once every time would not run out
        cp.attention(qd, kd, vd, mod="softcap", wait_limit_ns=1)
        torch.cuda.synchronize()
        try:
            cp.check_device_status(0)
        except cp.ChiaError as e:
            code = e.code
            break
    assert code == 5, "no wait ran out"
    torch.cuda.synchronize()
    assert int(ops._workspace(dev).abs().sum()) == 0
    check(cp.softcap_gemma2(qd, kd, vd), oracle.run_op("softcap_gemma2", q, k, v),
          "after a timeout")


# ------------------------------------------------------ split-KV decode path
def _decode_ref(op, q, k, v, okw, off):
    """Oracle of a decode-shaped call: the reference operator's mask, mod and
    normaliser with query row i at key position i + off (grouped K/V heads
    repeated per query head)."""
    from oracle import eager
    H, Hkv = q.shape[1], k.shape[1]
    kr, vr = (x.repeat_interleave(H // Hkv, dim=1) for x in (k, v))
    spec = {
        "softcap_gemma2": dict(norm="softmax", mod=lambda s, h, i, j: torch.tanh(s / 30.0) * 30.0),
        "bias_alibi": dict(norm="softmax",
                           mod=lambda s, h, i, j: s + okw["slopes"][h] * (j - (i + off)).float()),
        "temp_perhead": dict(norm="softmax", mod=lambda s, h, i, j: s * okw["temps"][h]),
        "sigmoid_attn": dict(norm="sigmoid", mod=lambda s, h, i, j: s + okw.get("bias", 0.0)),
        "relu_attn": dict(norm="relu", mod=None),
        "plain": dict(norm="softmax", mod=None),
    }[op]
    out = eager._eval(q, kr, vr, maskfn=lambda i, j: j <= i + off, **spec)
    return out * okw.get("out_scale", 1.0) if op == "relu_attn" else out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Sq,H,Hkv,Skv", [(1, 8, 1, 3000), (1, 4, 4, 777), (4, 8, 2, 2049),
                                          (2, 32, 2, 5000)])
@pytest.mark.parametrize("op", ["plain", "softcap_gemma2", "bias_alibi", "temp_perhead",
                                "sigmoid_attn", "relu_attn"])
def test_split_kv_decode_matches_oracle(cuda, op, Sq, H, Hkv, Skv, D, dtype):
    """Decode-shaped calls (rows per K/V head = H / H_kv * S_q <= 32) take the
    split-KV kernel: query row i sits at key position Skv - Sq + i (causal,
    bottom-right aligned), grouped K/V heads, every score modification."""
    off = Skv - Sq
    q, _, _ = gen(2, H, Sq, D, dtype, seed=Sq + H + D)
    _, k, v = gen(2, Hkv, Skv, D, dtype, seed=Skv + D)
    okw = {"bias_alibi": dict(slopes=cp.alibi_slopes_geometric(H)),
           "temp_perhead": dict(temps=1.0 / _tau(H)),
           "sigmoid_attn": dict(bias=-math.log(Skv)),
           "relu_attn": dict(out_scale=1.0 / Skv)}.get(op, {})
    kw = dict(norm={"sigmoid_attn": "sigmoid", "relu_attn": "relu"}.get(op, "softmax"),
              mod={"softcap_gemma2": "softcap", "bias_alibi": "alibi",
                   "temp_perhead": "temp"}.get(op, "none"),
              mask=cp.Mask(left=-1, right=off))
    if op == "bias_alibi":
        kw["head_param"] = okw["slopes"]
    if op == "temp_perhead":
        kw["head_param"] = okw["temps"]
    if op == "sigmoid_attn":
        kw["sig_bias"] = okw["bias"]
    if op == "relu_attn":
        kw["out_scale"] = okw["out_scale"]
    dev = torch.device("cuda", 0)
    out = cp.attention(q.to(dev), k.to(dev), v.to(dev), split_kv=True, **kw)
    torch.cuda.synchronize()
    check(out, _decode_ref(op, q, k, v, okw, off), f"{op} Sq={Sq} H={H}/{Hkv} Skv={Skv}")


@pytest.mark.parametrize("op,kw", [("bias_sliding_window", dict(window=100)),
                                   ("bias_local", dict(window=64)),
                                   ("bias_block_diagonal", dict(block=40)),
                                   ("bias_dilated", dict(dilation=3)),
                                   ("bias_prefix_lm", dict(prefix=20)),
                                   ("softcap_gemma2", dict(cap=50.0, causal=False))])
def test_split_kv_decode_masks(cuda, op, kw):
    """Every mask shape through the decode kernel, on rows 0..S_q-1 of the
    reference operators (top-left aligned, S_q < S_kv), against the oracle
    and against the tiled kernel."""
    H, Sq, Skv, D = 4, 30, 1500, 128   # 30 rows per K/V head: decode-shaped
    q, _, _ = gen(1, H, Sq, D, torch.bfloat16, seed=101)
    _, k, v = gen(1, H, Skv, D, torch.bfloat16, seed=102)
    dev = torch.device("cuda", 0)
    mask = cp.op_config(op, **kw)
    mod = "softcap" if op == "softcap_gemma2" else "none"
    extra = dict(softcap=kw["cap"]) if op == "softcap_gemma2" else {}
    out = cp.attention(q.to(dev), k.to(dev), v.to(dev), mask=mask, mod=mod, split_kv=True,
                       **extra)
    tiled = cp.attention(q.to(dev), k.to(dev), v.to(dev), mask=mask, mod=mod, split_kv=False,
                         **extra)
    torch.cuda.synchronize()
    from oracle import eager
    i_ = torch.arange(Sq).view(-1, 1)
    j_ = torch.arange(Skv).view(1, -1)
    band = torch.ones(Sq, Skv, dtype=torch.bool)
    if mask.left >= 0:
        band &= (i_ - j_) <= mask.left
    if mask.right >= 0:
        band &= (j_ - i_) <= mask.right
    if mask.block > 0:
        band &= (i_ // mask.block) == (j_ // mask.block)
    band &= ((i_ - j_) % mask.dilation) == 0
    vis = band | (j_ < mask.prefix)
    modf = (lambda s, h, i, j: torch.tanh(s / kw["cap"]) * kw["cap"]) if extra else None
    ref = torch.nan_to_num(eager._eval(q, k, v, maskfn=lambda i, j: vis[i.flatten()][:, j.flatten()],
                                       mod=modf), nan=0.0)
    check(out, ref, f"{op} decode")
    check(tiled, ref, f"{op} tiled")


def test_split_kv_decode_long_gqa_and_lse(cuda):
    """One new token per sequence over 8192 cached keys, 32 query heads on 4
    K/V heads (GQA 8:1): sampled heads against the oracle, and the decode
    kernel's log-sum-exp against the oracle's."""
    B, H, Hkv, Skv, D = 4, 32, 4, 8192, 128
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(111)
    q = torch.randn(B, H, 1, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(B, Hkv, Skv, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(B, Hkv, Skv, D, generator=g, device=dev).to(torch.bfloat16)
    out, lse = cp.attention(q, k, v, mask=cp.Mask(left=-1, right=Skv - 1), return_lse=True)
    torch.cuda.synchronize()
    for b, h in ((0, 0), (1, 9), (3, 31)):
        hk = h // (H // Hkv)
        qs, ks, vs = q[b:b + 1, h:h + 1].cpu(), k[b:b + 1, hk:hk + 1].cpu(), v[b:b + 1, hk:hk + 1].cpu()
        ref, ref_lse = oracle.run_op_lse("softcap_gemma2", qs, ks, vs, cap=1e30, causal=False)
        check(out[b:b + 1, h:h + 1], ref, f"head ({b},{h})")
        assert abs(lse[b, h, 0].item() - ref_lse[0, 0, 0].item()) < 1e-3
