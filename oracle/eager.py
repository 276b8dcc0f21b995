"""fp32 CPU restatement of the reference's eager attention functions.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference semantics (JoshiP-commits/CHIA_proj ``extra_bench.py:32-62``):

* ``s = (q @ k^T) * SC`` with ``SC = 1/sqrt(D)``            (``extra_bench.py:33,39``)
* optional score modification ``mod(s)``                     (``extra_bench.py:40``)
* mask ``ok(i, j)``, default causal ``j <= i``                (``extra_bench.py:41``)
* normaliser: softmax over ``masked_fill(~ok, -inf)``; or
  ``sigmoid(s) * ok``; or ``relu(s) * ok``                     (``extra_bench.py:42-44``)
  -- the sigmoid mask is applied AFTER the nonlinearity, as in the corrected
  reference ``sigmoid_fix.py:34-40`` (the pre-fix ``synth10.py:48`` form is
  not used)
* ``p @ v``                                                   (``extra_bench.py:45``)
* ALiBi: ``s + slope_h * (j - i)`` then causal softmax         (``extra_bench.py:47-50``)

The ten variants and their reference masks / mods are listed in
``extra_bench.py:51-62``. Everything here runs in fp32 (the reference's
``DT`` set to ``torch.float32``), on CPU, one (b, h) pair and one block of
query rows at a time so that large sequence lengths fit in memory.

Each public function keeps the reference defaults and adds the parameters
the benchmark configurations vary (keyword-only).
"""

from __future__ import annotations

import math
from typing import Callable, Dict, Optional

import torch
import torch.nn.functional as F

__all__ = ["OPS", "run_op", "run_op_lse", "reference_masks", "visible_pairs_dense"]

# When set (by run_op_lse), _eval stores each softmax row's natural
# log-sum-exp of the modified, masked scores here, [B, H, S_q].
_lse_sink: Optional[torch.Tensor] = None


# ---------------------------------------------------------------------------
# masks, written as the reference writes them (extra_bench.py:55-61)
# ---------------------------------------------------------------------------
def reference_masks(window: int = 256, block: int = 512, prefix: int = 256,
                    dilation: int = 4, causal_block: bool = True,
                    local: int = 256) -> Dict[str, Callable]:
    """Boolean mask lambdas ``ok(i, j)`` of the reference (``extra_bench.py:55-61``).

    ``i`` is a column vector of query indices and ``j`` a row vector of key
    indices; defaults are the reference's hardcoded values.
    """
    def causal(i, j):
        return j <= i

    def dilated(i, j):            # extra_bench.py:56
        return (j <= i) & (((i - j) % dilation) == 0)

    def local_(i, j):             # extra_bench.py:57
        return (i - j).abs() < local

    def block_diag(i, j):         # extra_bench.py:58
        same = (torch.div(i, block, rounding_mode="floor")
                == torch.div(j, block, rounding_mode="floor"))
        return (same & (j <= i)) if causal_block else same

    def prefix_lm(i, j):          # extra_bench.py:59
        return (j <= i) | (j < prefix)

    def sliding(i, j):            # extra_bench.py:61
        return (j <= i) & ((i - j) < window)

    def full(i, j):
        return torch.ones(i.shape[0], j.shape[1], dtype=torch.bool)

    return {"causal": causal, "full": full, "bias_dilated": dilated,
            "bias_local": local_, "bias_block_diagonal": block_diag,
            "bias_prefix_lm": prefix_lm, "bias_sliding_window": sliding}


def _rows(i0: int, i1: int) -> torch.Tensor:
    return torch.arange(i0, i1).view(-1, 1)


def _cols(n: int) -> torch.Tensor:
    return torch.arange(n).view(1, -1)


# ---------------------------------------------------------------------------
# one generic fp32 evaluator: s -> mod -> mask -> normaliser -> p @ v
# ---------------------------------------------------------------------------
def _eval(q, k, v, *, maskfn, norm="softmax", mod=None, scale=None,
          row_block=1024):
    """Evaluate one attention variant in fp32 on CPU.

    ``mod(s, h, i, j)`` receives the fp32 scaled scores of head ``h`` for query
    rows ``i`` (column vector) and keys ``j`` (row vector). ``maskfn(i, j)``
    returns the visibility mask. ``norm`` is ``"softmax"`` (masked_fill
    -inf, fp32 softmax: ``extra_bench.py:42``), ``"sigmoid"`` (sigmoid then
    multiply by the mask: ``sigmoid_fix.py:37-39``) or ``"relu"``
    (``extra_bench.py:44``).
    """
    if q.dim() != 4:
        raise ValueError("expected [B, H, S, D] tensors")
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    sc = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    qf, kf, vf = q.float(), k.float(), v.float()
    out = torch.empty(B, H, Sq, v.shape[-1], dtype=torch.float32)
    j = _cols(Skv)
    for b in range(B):
        for h in range(H):
            kt = kf[b, h].transpose(0, 1)
            for i0 in range(0, Sq, row_block):
                i1 = min(Sq, i0 + row_block)
                i = _rows(i0, i1)
                s = (qf[b, h, i0:i1] @ kt) * sc
                if mod is not None:
                    s = mod(s, h, i, j)
                ok = maskfn(i, j)
                if norm == "softmax":
                    sm = s.masked_fill(~ok, float("-inf"))
                    p = torch.softmax(sm, -1)
                    if _lse_sink is not None:
                        _lse_sink[b, h, i0:i1] = torch.logsumexp(sm, -1).detach()
                elif norm == "sigmoid":
                    p = torch.sigmoid(s) * ok.float()
                elif norm == "relu":
                    p = F.relu(s) * ok.float()
                else:
                    raise ValueError(norm)
                out[b, h, i0:i1] = p @ vf[b, h]
    return out


# ---------------------------------------------------------------------------
# the ten reference operators (extra_bench.py:51-62), fp32
# ---------------------------------------------------------------------------
def softcap_gemma2(q, k, v, *, cap: float = 30.0, causal: bool = True):
    """``tanh(s/cap)*cap`` then softmax; reference: cap 30, causal (``extra_bench.py:60``)."""
    m = reference_masks()
    return _eval(q, k, v, maskfn=m["causal"] if causal else m["full"],
                 mod=lambda s, h, i, j: torch.tanh(s / cap) * cap)


def bias_sliding_window(q, k, v, *, window: int = 256):
    """Causal window ``(j<=i)&(i-j<window)`` (``extra_bench.py:61``)."""
    return _eval(q, k, v, maskfn=reference_masks(window=window)["bias_sliding_window"])


def bias_local(q, k, v, *, window: int = 256):
    """Bidirectional band ``|i-j|<window`` (``extra_bench.py:57``)."""
    return _eval(q, k, v, maskfn=reference_masks(local=window)["bias_local"])


def default_alibi_slopes(H: int) -> torch.Tensor:
    """Reference slopes ``h+1`` as fp32 (``extra_bench.py:36``)."""
    return torch.arange(1, H + 1, dtype=torch.float32)


def bias_alibi(q, k, v, *, slopes: Optional[torch.Tensor] = None):
    """``s + slope_h*(j-i)``, causal softmax (``extra_bench.py:47-50``)."""
    H = q.shape[1]
    sl = default_alibi_slopes(H) if slopes is None else slopes.detach().float().cpu()
    return _eval(q, k, v, maskfn=reference_masks()["causal"],
                 mod=lambda s, h, i, j: s + sl[h] * (j - i).float())


def bias_block_diagonal(q, k, v, *, block: int = 512, causal: bool = True):
    """Same-block mask, causal inside a block by default (``extra_bench.py:58``)."""
    return _eval(q, k, v, maskfn=reference_masks(block=block, causal_block=causal)[
        "bias_block_diagonal"])


def bias_dilated(q, k, v, *, dilation: int = 4):
    """``(j<=i)&((i-j)%dilation==0)`` (``extra_bench.py:56``)."""
    return _eval(q, k, v, maskfn=reference_masks(dilation=dilation)["bias_dilated"])


def bias_prefix_lm(q, k, v, *, prefix: int = 256):
    """``(j<=i)|(j<prefix)`` (``extra_bench.py:59``)."""
    return _eval(q, k, v, maskfn=reference_masks(prefix=prefix)["bias_prefix_lm"])


def default_temps(H: int) -> torch.Tensor:
    """Reference per-head multipliers ``0.5+h/H`` (``extra_bench.py:35``)."""
    return 0.5 + torch.arange(H, dtype=torch.float32) / H


def temp_perhead(q, k, v, *, temps: Optional[torch.Tensor] = None):
    """``s*TEMP[h]``, causal softmax (``extra_bench.py:35,54``).

    ``temps`` multiplies the scaled logits, as the reference's ``TEMP`` does;
    a temperature ``tau_h`` dividing the logits is ``temps = 1/tau``.
    """
    H = q.shape[1]
    t = default_temps(H) if temps is None else temps.detach().float().cpu()
    return _eval(q, k, v, maskfn=reference_masks()["causal"],
                 mod=lambda s, h, i, j: s * t[h])


def sigmoid_attn(q, k, v, *, causal: bool = True, bias: float = 0.0):
    """``sigmoid(s+bias)*mask`` -- mask after the sigmoid (``sigmoid_fix.py:34-40``)."""
    m = reference_masks()
    mod = None if bias == 0.0 else (lambda s, h, i, j: s + bias)
    return _eval(q, k, v, maskfn=m["causal"] if causal else m["full"],
                 norm="sigmoid", mod=mod)


def relu_attn(q, k, v, *, causal: bool = True, out_scale: float = 1.0):
    """``relu(s)*mask @ v``, times ``out_scale`` (``extra_bench.py:44``)."""
    m = reference_masks()
    out = _eval(q, k, v, maskfn=m["causal"] if causal else m["full"], norm="relu")
    return out * out_scale if out_scale != 1.0 else out


OPS = {
    "sigmoid_attn": sigmoid_attn,
    "relu_attn": relu_attn,
    "temp_perhead": temp_perhead,
    "bias_alibi": bias_alibi,
    "bias_dilated": bias_dilated,
    "bias_local": bias_local,
    "bias_block_diagonal": bias_block_diagonal,
    "bias_prefix_lm": bias_prefix_lm,
    "softcap_gemma2": softcap_gemma2,
    "bias_sliding_window": bias_sliding_window,
}


def run_op(op: str, q, k, v, **params) -> torch.Tensor:
    """Run reference operator ``op`` in fp32 on CPU; returns fp32 ``[B,H,S,D]``."""
    return OPS[op](q.cpu(), k.cpu(), v.cpu(), **params)


def run_op_lse(op: str, q, k, v, **params):
    """``run_op`` plus the natural log-sum-exp of every softmax row's
    modified, masked scores (``-inf`` where a row sees no key), fp32
    ``[B, H, S_q]``. Not part of the reference, whose eager functions return
    the output only; it pins the forward's LSE output, which the backward
    pass reads."""
    global _lse_sink
    B, H, Sq, _ = q.shape
    _lse_sink = torch.full((B, H, Sq), float("-inf"))
    try:
        out = run_op(op, q, k, v, **params)
        return out, _lse_sink
    finally:
        _lse_sink = None


def run_varlen(op: str, q, k, v, cu_seqlens, **params) -> torch.Tensor:
    """Packed variable-length sequences: ``q, k, v`` are ``[1, H, S, D]`` whose
    tokens are the concatenated sequences, sequence ``s`` at
    ``[cu_seqlens[s], cu_seqlens[s+1])``. No counterpart in the reference (its
    operators take one length per batch); the meaning is the reference
    operator applied to each sequence on its own, which is what this does."""
    cu = [int(x) for x in (cu_seqlens.tolist() if hasattr(cu_seqlens, "tolist") else cu_seqlens)]
    out = torch.zeros(q.shape, dtype=torch.float32)
    for a, b in zip(cu, cu[1:]):
        if b > a:
            out[:, :, a:b] = run_op(op, q[:, :, a:b], k[:, :, a:b], v[:, :, a:b], **params)
    return out


def visible_pairs_dense(maskfn: Callable, S: int) -> int:
    """Count visible (i, j) pairs of a reference mask by dense evaluation (small S)."""
    i = _rows(0, S)
    j = _cols(S)
    return int(maskfn(i, j).sum().item())
