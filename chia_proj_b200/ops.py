"""The ten attention operators, with the reference's eager call signatures.

Each function takes ``q, k, v`` of shape ``[B, H, S, D]`` on a B200 and
returns ``out`` of the same shape and dtype, exactly like the reference's
eager closures in ``build_refs()`` (JoshiP-commits/CHIA_proj
``extra_bench.py:32-62``; corrected sigmoid ``sigmoid_fix.py:34-40``) and its
plugin entry point ``launch_kernel(q, k, v)`` (``extra_bench.py:24-27``).
Keyword arguments default to the reference's hardcoded values; the benchmark
configurations change them (softcap 50 non-causal, geometric ALiBi slopes,
block 256, prefix 1024, sigmoid bias -log S, ReLU scale 1/S, ...).

All computation happens in ``libchia_attn.so`` (one sm_100a kernel launch per
call, on the current CUDA stream). There is no CPU or PyTorch fallback: CPU
tensors raise, a missing library raises.

Numerics: q.k and P.V run on the tensor cores with fp32 accumulation; the
score modification, mask and normaliser run in fp32; P is rounded to the
input dtype before P.V, as the reference's ``p.to(DT) @ v`` does
(``extra_bench.py:45``). fp32 inputs are accepted for signature
and computed on the tensor cores with 16-bit operands and fp32 accumulation:
fp16 operands (a 10-bit mantissa, the precision of a TF32 MMA) when every
input element and every score fits fp16's range, else bf16 operands;
``compute_dtype`` chooses explicitly. The output is returned in fp32.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Dict, Optional, Sequence, Union

import torch

from . import _native as N

__all__ = [
    "Mask", "CAUSAL", "FULL", "attention", "OPS", "op_config", "visible_pairs",
    "softcap_gemma2", "bias_sliding_window", "bias_local", "bias_alibi",
    "bias_block_diagonal", "bias_dilated", "bias_prefix_lm", "temp_perhead",
    "sigmoid_attn", "relu_attn", "alibi_slopes_geometric", "reference_alibi_slopes",
    "reference_temps", "check_device_status", "attention_backward",
]


@dataclass(frozen=True)
class Mask:
    """Visibility of key j for query i (``include/chia_attn.h``).

    ``vis = j < prefix or (i-j <= left [left>=0] and j-i <= right [right>=0]
    and same block [block>0] and (i-j) % dilation == 0)``.
    """

    left: int = -1
    right: int = 0
    block: int = 0
    prefix: int = 0
    dilation: int = 1

    def validate(self) -> "Mask":
        if self.left < -1 or self.right < -1 or self.block < 0 or self.prefix < 0 \
                or self.dilation < 1:
            raise ValueError(f"invalid mask {self}")
        return self


CAUSAL = Mask(left=-1, right=0)
FULL = Mask(left=-1, right=-1)

_NORMS = {"softmax": N.NORM_SOFTMAX, "sigmoid": N.NORM_SIGMOID, "relu": N.NORM_RELU}
_MODS = {"none": N.MOD_NONE, "softcap": N.MOD_SOFTCAP, "alibi": N.MOD_ALIBI,
         "temp": N.MOD_TEMP}

_status_words: Dict[int, torch.Tensor] = {}
_workspaces: Dict[tuple, torch.Tensor] = {}
_param_cache: Dict[tuple, torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status_words.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = t
    return t


def _workspace(device: torch.device, stream: Optional[int] = None) -> torch.Tensor:
    """Scheduler workspace of one (device, stream) pair (zero-filled once;
    every kernel leaves it zeroed).

    Launches on one stream run in order, so they may share a workspace;
    launches on two streams may overlap on the GPU and would race on the
    scheduler's counters, so each stream gets its own.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = torch.cuda.current_stream(idx).cuda_stream
    key = (idx, int(stream))
    t = _workspaces.get(key)
    if t is None:
        t = torch.zeros(N.WORKSPACE_BYTES // 4, dtype=torch.int32,
                        device=torch.device("cuda", idx))
        _workspaces[key] = t
    return t


_decode_workspaces: Dict[tuple, torch.Tensor] = {}


def _decode_workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Workspace of the split-KV decode path for one (device, stream): zero-
    filled when (re)allocated, left with zeroed counters by every call."""
    key = (device.index, int(stream))
    t = _decode_workspaces.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _decode_workspaces[key] = t
    return t


DECODE_MAX_ROWS = 32  # (H / H_kv) * S_q of a decode-shaped call


def check_device_status(device: Optional[Union[int, torch.device]] = None) -> None:
    """Synchronise ``device`` and raise if any kernel there reported an error.

    Kernels OR error codes (a bounded wait that expired) into a per-device
    status word instead of trapping; this reads and clears it.
    """
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    w = _status_word(dev)
    code = int(w.item())
    if code:
        w.zero_()
        raise N.ChiaError(code, "reported by a kernel on " + str(dev))


def _param_tensor(values, H: int, device: torch.device) -> torch.Tensor:
    if isinstance(values, torch.Tensor):
        t = values.detach().to(device=device, dtype=torch.float32).contiguous()
    else:
        t = torch.tensor(list(values), dtype=torch.float32, device=device)
    if t.numel() != H:
        raise ValueError(f"per-head parameter must have {H} entries, got {t.numel()}")
    return t


def reference_alibi_slopes(H: int) -> torch.Tensor:
    """ALiBi slopes of the reference, ``h+1`` (``extra_bench.py:36``)."""
    return torch.arange(1, H + 1, dtype=torch.float32)


def alibi_slopes_geometric(H: int) -> torch.Tensor:
    """Geometric ALiBi slopes ``2^(-8(h+1)/H)`` (the benchmark configuration)."""
    return torch.pow(2.0, -8.0 * (torch.arange(H, dtype=torch.float32) + 1) / H)


def reference_temps(H: int) -> torch.Tensor:
    """Per-head multipliers of the reference, ``0.5+h/H`` (``extra_bench.py:35``)."""
    return 0.5 + torch.arange(H, dtype=torch.float32) / H


def _cached_default(kind: str, H: int, device: torch.device) -> torch.Tensor:
    key = (kind, H, str(device))
    t = _param_cache.get(key)
    if t is None:
        src = reference_alibi_slopes(H) if kind == "alibi" else reference_temps(H)
        t = src.to(device)
        _param_cache[key] = t
    return t


def _prep(x: torch.Tensor) -> torch.Tensor:
    """Make a tensor TMA-compatible: unit last stride, 16-byte aligned rows."""
    if x.stride(-1) != 1 or any(s % 8 for s in x.stride()[:-1]) or x.data_ptr() % 16:
        x = x.contiguous()
    return x


_FP16_MAX = 65504.0


def _fp32_operand_dtype(q, k, v, norm: str, scale) -> torch.dtype:
    """Operand type for fp32 inputs: fp16 when nothing the kernel rounds to
    16 bits can leave fp16's range, else bf16. The inputs must fit; so must P,
    which is at most 1 for softmax and sigmoid and at most
    max|q| max|k| D scale for ReLU (the output scale is applied after P.V)."""
    amax = torch.stack([torch.linalg.vector_norm(t.detach(), float("inf"))
                        for t in (q, k, v)]).cpu()
    if not bool(torch.isfinite(amax).all()) or float(amax.max()) > _FP16_MAX:
        return torch.bfloat16
    if norm == "relu":
        D = q.shape[-1]
        sc = abs(scale) if scale is not None else 1.0 / math.sqrt(D)
        if float(amax[0]) * float(amax[1]) * D * sc > _FP16_MAX:
            return torch.bfloat16
    return torch.float16


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
              norm: str = "softmax", mod: str = "none", mask: Mask = CAUSAL,
              scale: Optional[float] = None, softcap: float = 30.0,
              head_param: Optional[Union[torch.Tensor, Sequence[float]]] = None,
              sig_bias: float = 0.0, out_scale: float = 1.0,
              out: Optional[torch.Tensor] = None, schedule: str = "dynamic",
              cu_seqlens=None, return_lse: bool = False, wait_limit_ns: int = 0,
              split_kv: Optional[bool] = None,
              compute_dtype: Optional[torch.dtype] = None):
    """Generic forward attention: ``norm(mask(mod(q.k * scale))) @ v``.

    ``q, k, v``: CUDA tensors ``[B, H, S, D]`` (bf16 / fp16 / fp32), ``D`` in
    {64, 128}. fp32 inputs are computed with 16-bit tensor-core operands and
    fp32 accumulation, and the output is fp32: ``compute_dtype`` (fp16 or
    bf16) names the operand type; ``None`` takes fp16 (10 mantissa bits, as
    a TF32 MMA keeps) when the inputs and the largest possible score fit its
    range, else bf16. ``k`` and ``v`` may have ``H_kv`` heads with
    ``H % H_kv == 0`` (grouped-query attention: query head ``h`` reads K/V
    head ``h // (H // H_kv)``). ``head_param``: ALiBi slopes (``mod="alibi"``)
    or logit multipliers (``mod="temp"``), one per head. ``schedule``:
    ``"dynamic"`` balances work units over the SMs with a workspace per
    (device, stream); ``"static"`` assigns them round-robin and uses none.
    ``cu_seqlens``: packed variable-length sequences. ``q, k, v`` hold a
    batch of 1 whose ``S`` tokens are the concatenated sequences, with
    sequence ``s`` at tokens ``[cu_seqlens[s], cu_seqlens[s+1])``; a query
    sees keys of its own sequence only (then ``mask``, which may not use a
    block, prefix or dilation). A list or CPU tensor is checked and copied to
    the device; a CUDA int32 tensor is used as given.
    ``return_lse``: also return the natural log-sum-exp of every row's
    modified, masked scores, fp32 ``[B, H, S]`` (softmax only; ``-inf`` for a
    row that sees no key) -- what the backward pass needs.
    ``wait_limit_ns``: limit of each in-kernel wait (0 = 2 s). A wait that
    runs out is reported by ``check_device_status``; tests use tiny values to
    exercise that path.
    ``split_kv``: decode-shaped calls -- at most 32 rows per K/V head
    (``(H // H_kv) * S_q``) and ``S_q <= 64`` -- run on the split-KV decode
    kernel, which spreads the keys of each K/V head over many SMs; ``None``
    chooses it for those shapes, ``False`` forces the tiled kernel, ``True``
    requires the decode kernel.
    """
    if (torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad
                                        for t in (q, k, v))):
        if out is not None or cu_seqlens is not None:
            raise ValueError("out= and cu_seqlens= do not support gradients")
        o, lse = _AttentionFn.apply(q, k, v, norm, mod, mask, scale, softcap, head_param,
                                    sig_bias, out_scale)
        return (o, lse) if return_lse else o
    if schedule not in ("dynamic", "static"):
        raise ValueError(f"unknown schedule {schedule!r}")
    if norm not in _NORMS or mod not in _MODS:
        raise ValueError(f"unknown norm/mod {norm!r}/{mod!r}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor) or t.dim() != 4:
            raise ValueError(f"{name} must be a [B, H, S, D] tensor")
        if t.device.type != "cuda":
            raise RuntimeError(f"{name} is on {t.device}: the library runs on CUDA only "
                               "(no CPU fallback)")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share a dtype")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on one device")
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    if (k.shape != (B, Hkv, k.shape[2], D) or v.shape != k.shape or Hkv < 1
            or H % Hkv != 0):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if D not in (64, 128):
        raise ValueError(f"head_dim {D} unsupported (64 or 128)")
    mask = mask.validate()
    if return_lse and norm != "softmax":
        raise ValueError("return_lse needs norm='softmax'")
    if wait_limit_ns < 0:
        raise ValueError("wait_limit_ns must be >= 0")
    in_dtype = q.dtype
    if in_dtype == torch.float32:
        cdt = (compute_dtype if compute_dtype is not None
               else _fp32_operand_dtype(q, k, v, norm, scale))
        if cdt not in (torch.float16, torch.bfloat16):
            raise ValueError("compute_dtype must be torch.float16 or torch.bfloat16")
        q, k, v = q.to(cdt), k.to(cdt), v.to(cdt)
    elif in_dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"dtype {in_dtype} unsupported")
    elif compute_dtype is not None and compute_dtype != in_dtype:
        raise ValueError("compute_dtype applies to fp32 inputs only")
    q, k, v = _prep(q), _prep(k), _prep(v)
    dev = q.device
    if out is None or in_dtype == torch.float32:
        o = torch.empty(B, H, S, D, dtype=q.dtype, device=dev)
    else:
        if out.shape != q.shape or out.dtype != q.dtype or out.device != dev:
            raise ValueError("out must match q in shape, dtype and device")
        o = out
        if o.stride(-1) != 1 or any(s % 8 for s in o.stride()[:-1]) or o.data_ptr() % 16:
            raise ValueError("out must have unit last stride and 16-byte aligned rows")

    seg = None
    if cu_seqlens is not None:
        if B != 1 or k.shape[2] != S:
            raise ValueError("packed sequences need a batch of 1 and S_q == S_kv")
        if mask.block or mask.prefix or mask.dilation != 1:
            raise ValueError("packed sequences take window and causal masks only")
        cu = cu_seqlens if isinstance(cu_seqlens, torch.Tensor) else torch.tensor(cu_seqlens)
        if cu.dim() != 1 or cu.numel() < 2:
            raise ValueError("cu_seqlens must be 1-D with at least two offsets")
        if cu.device.type == "cuda":
            if cu.dtype != torch.int32 or cu.device != dev:
                raise ValueError("a CUDA cu_seqlens must be int32 on the device of q")
            seg = cu.contiguous()
        else:
            c = [int(x) for x in cu.tolist()]
            if c[0] != 0 or c[-1] != S or any(b < a for a, b in zip(c, c[1:])):
                raise ValueError(f"cu_seqlens must rise from 0 to S={S}")
            seg = torch.tensor(c, dtype=torch.int32, device=dev)

    hp = None
    if mod in ("alibi", "temp"):
        hp = (_cached_default(mod, H, dev) if head_param is None
              else _param_tensor(head_param, H, dev))

    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.dtype = N.DTYPE_BF16 if q.dtype == torch.bfloat16 else N.DTYPE_F16
    p.head_dim = D
    p.norm = _NORMS[norm]
    p.mod = _MODS[mod]
    p.batch, p.heads, p.seqlen_q, p.seqlen_kv = B, H, S, k.shape[2]
    p.heads_kv = Hkv
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    for field, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", o)):
        getattr(p, field)[:] = t.stride()[:3]
    p.scale = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    p.softcap = float(softcap)
    p.sig_bias = float(sig_bias)
    p.out_scale = float(out_scale)
    p.head_param = hp.data_ptr() if hp is not None else None
    p.win_left, p.win_right = mask.left, mask.right
    p.block, p.prefix, p.dilation = mask.block, mask.prefix, mask.dilation
    p.status = _status_word(dev).data_ptr()
    if seg is not None:
        p.seq_offsets = seg.data_ptr()
        p.num_seqs = seg.numel() - 1
    lse = None
    if return_lse:
        lse = torch.empty(B, H, S, dtype=torch.float32, device=dev)
        p.lse = lse.data_ptr()
    p.wait_limit_ns = int(wait_limit_ns)

    decode_shape = (cu_seqlens is None and (H // Hkv) * S <= DECODE_MAX_ROWS and S <= 64)
    if split_kv and not decode_shape:
        raise ValueError("split_kv=True needs (H // H_kv) * S_q <= 32, S_q <= 64 and no "
                         "cu_seqlens")
    use_decode = decode_shape if split_kv is None else bool(split_kv)

    lib = N.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        if use_decode:
            nbytes = lib.chia_attn_decode_workspace_bytes(ctypes.byref(p))
            if nbytes < 0:
                raise ValueError("not a decode-shaped call")
            ws = _decode_workspace(dev, stream, nbytes)
            code = lib.chia_attn_decode(ctypes.byref(p), ctypes.c_void_p(ws.data_ptr()),
                                        ws.numel(), ctypes.c_void_p(stream))
            if code:  # the message is formatted only on failure (host time per call)
                N.check(code, f"chia_attn_decode(norm={norm}, mod={mod}, mask={mask}, "
                              f"q={tuple(q.shape)}, k={tuple(k.shape)})")
            o = o.float() if in_dtype == torch.float32 else o
            return (o, lse) if return_lse else o
        # one workspace per (device, stream): see _workspace
        p.workspace = _workspace(dev, stream).data_ptr() if schedule == "dynamic" else None
        code = lib.chia_attn_fwd(ctypes.byref(p), ctypes.c_void_p(stream))
        if code:  # the message is formatted only on failure (host time per call)
            N.check(code, f"chia_attn_fwd(norm={norm}, mod={mod}, mask={mask}, "
                          f"shape={tuple(q.shape)})")
    o = o.float() if in_dtype == torch.float32 else o
    return (o, lse) if return_lse else o


# ---------------------------------------------------------------------------
# backward pass
# ---------------------------------------------------------------------------
_bwd_workspaces: Dict[tuple, torch.Tensor] = {}


def _params_for(q, k, v, o, *, norm, mod, mask, scale, softcap, hp, sig_bias, out_scale,
                lse=None) -> "N.AttnParams":
    B, H, S, D = q.shape
    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.dtype = N.DTYPE_BF16 if q.dtype == torch.bfloat16 else N.DTYPE_F16
    p.head_dim = D
    p.norm, p.mod = _NORMS[norm], _MODS[mod]
    p.batch, p.heads, p.seqlen_q, p.seqlen_kv = B, H, S, k.shape[2]
    p.heads_kv = k.shape[1]
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    for field, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", o)):
        getattr(p, field)[:] = t.stride()[:3]
    p.scale = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    p.softcap, p.sig_bias, p.out_scale = float(softcap), float(sig_bias), float(out_scale)
    p.head_param = hp.data_ptr() if hp is not None else None
    p.win_left, p.win_right = mask.left, mask.right
    p.block, p.prefix, p.dilation = mask.block, mask.prefix, mask.dilation
    p.status = _status_word(q.device).data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    return p


def attention_backward(dout, q, k, v, out, lse, *, norm="softmax", mod="none", mask=CAUSAL,
                       scale=None, softcap=30.0, head_param=None, sig_bias=0.0, out_scale=1.0):
    """Gradients ``(dq, dk, dv)`` of ``attention(q, k, v, ...)`` given the
    upstream gradient ``dout``, the forward's output ``out`` and (softmax)
    its log-sum-exp ``lse`` (``attention(..., return_lse=True)``). One call
    of ``chia_attn_bwd``; ``dk``, ``dv`` have the K/V heads of ``k``, ``v``."""
    q, k, v, out, dout = (_prep(t) for t in (q, k, v, out, dout))
    dev = q.device
    if not (q.dtype == k.dtype == v.dtype == out.dtype == dout.dtype):
        raise ValueError("q, k, v, out, dout must share a dtype")
    if norm == "softmax" and lse is None:
        raise ValueError("the softmax backward needs the forward's lse")
    hp = None
    if mod in ("alibi", "temp"):
        hp = (_cached_default(mod, q.shape[1], dev) if head_param is None
              else _param_tensor(head_param, q.shape[1], dev))
    p = _params_for(q, k, v, out, norm=norm, mod=mod, mask=mask.validate(), scale=scale,
                    softcap=softcap, hp=hp, sig_bias=sig_bias, out_scale=out_scale,
                    lse=lse.contiguous() if lse is not None else None)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    g = N.AttnGrads()
    g.dout = dout.data_ptr()
    g.dout_stride[:] = dout.stride()[:3]
    g.dq, g.dk, g.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    g.dq_stride[:] = dq.stride()[:3]
    g.dk_stride[:] = dk.stride()[:3]
    g.dv_stride[:] = dv.stride()[:3]
    lib = N.load()
    nbytes = lib.chia_attn_bwd_workspace_bytes(ctypes.byref(p))
    if nbytes < 0:
        raise ValueError("invalid backward parameters")
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        key = (dev.index, int(stream))
        ws = _bwd_workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            _bwd_workspaces[key] = ws
        code = lib.chia_attn_bwd(ctypes.byref(p), ctypes.byref(g), ctypes.c_void_p(ws.data_ptr()),
                                 ws.numel(), ctypes.c_void_p(stream))
        if code:  # the message is formatted only on failure
            N.check(code, f"chia_attn_bwd(norm={norm}, mod={mod}, mask={mask}, "
                          f"shape={tuple(q.shape)})")
    return dq, dk, dv


class _AttentionFn(torch.autograd.Function):
    """Autograd for ``attention``: the forward kernel (with the log-sum-exp
    for softmax), the backward kernel for the gradients of q, k and v.
    Per-head parameters and scalars are not differentiated."""

    @staticmethod
    def forward(ctx, q, k, v, norm, mod, mask, scale, softcap, head_param, sig_bias, out_scale):
        kw = dict(norm=norm, mod=mod, mask=mask, scale=scale, softcap=softcap,
                  head_param=head_param, sig_bias=sig_bias, out_scale=out_scale)
        with torch.no_grad():
            if norm == "softmax":
                o, lse = attention(q, k, v, return_lse=True, split_kv=False, **kw)
            else:
                o, lse = attention(q, k, v, split_kv=False, **kw), None
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.kw = kw
        ctx.mark_non_differentiable(*(x for x in (lse,) if x is not None))
        return o, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = attention_backward(dout.to(o.dtype), q, k, v, o, lse, **ctx.kw)
        return dq, dk, dv, None, None, None, None, None, None, None, None


# ---------------------------------------------------------------------------
# the ten reference operators (extra_bench.py:51-62)
# ---------------------------------------------------------------------------
def softcap_gemma2(q, k, v, *, cap: float = 30.0, causal: bool = True,
                   scale: Optional[float] = None, cu_seqlens=None):
    """Gemma-2 softcap: ``softmax(cap*tanh(s/cap))`` (``extra_bench.py:60``)."""
    return attention(q, k, v, mod="softcap", softcap=cap, mask=CAUSAL if causal else FULL,
                     scale=scale, cu_seqlens=cu_seqlens)


def bias_sliding_window(q, k, v, *, window: int = 256, scale: Optional[float] = None,
                        cu_seqlens=None):
    """Causal window ``(j<=i)&(i-j<window)`` (``extra_bench.py:61``)."""
    if window < 1:
        raise ValueError("window must be >= 1")
    return attention(q, k, v, mask=Mask(left=window - 1, right=0), scale=scale,
                     cu_seqlens=cu_seqlens)


def bias_local(q, k, v, *, window: int = 256, scale: Optional[float] = None, cu_seqlens=None):
    """Bidirectional band ``|i-j|<window`` (``extra_bench.py:57``)."""
    if window < 1:
        raise ValueError("window must be >= 1")
    return attention(q, k, v, mask=Mask(left=window - 1, right=window - 1), scale=scale,
                     cu_seqlens=cu_seqlens)


def bias_alibi(q, k, v, *, slopes=None, scale: Optional[float] = None, cu_seqlens=None):
    """ALiBi ``s + slope_h*(j-i)``, causal (``extra_bench.py:47-50``); default slopes h+1."""
    return attention(q, k, v, mod="alibi", head_param=slopes, mask=CAUSAL, scale=scale,
                     cu_seqlens=cu_seqlens)


def bias_block_diagonal(q, k, v, *, block: int = 512, causal: bool = True,
                        scale: Optional[float] = None):
    """Same-block mask, causal inside blocks by default (``extra_bench.py:58``)."""
    if block < 1:
        raise ValueError("block must be >= 1")
    return attention(q, k, v, mask=Mask(left=-1, right=0 if causal else -1, block=block),
                     scale=scale)


def bias_dilated(q, k, v, *, dilation: int = 4, scale: Optional[float] = None):
    """``(j<=i)&((i-j)%dilation==0)`` (``extra_bench.py:56``)."""
    if dilation < 1:
        raise ValueError("dilation must be >= 1")
    return attention(q, k, v, mask=Mask(left=-1, right=0, dilation=dilation), scale=scale)


def bias_prefix_lm(q, k, v, *, prefix: int = 256, scale: Optional[float] = None):
    """``(j<=i)|(j<prefix)`` (``extra_bench.py:59``)."""
    if prefix < 0:
        raise ValueError("prefix must be >= 0")
    return attention(q, k, v, mask=Mask(left=-1, right=0, prefix=prefix), scale=scale)


def temp_perhead(q, k, v, *, temps=None, scale: Optional[float] = None, cu_seqlens=None):
    """``s*TEMP[h]``, causal (``extra_bench.py:35,54``); default TEMP ``0.5+h/H``.

    ``temps`` multiplies the logits like the reference's TEMP; a temperature
    tau dividing them is ``temps = 1/tau``.
    """
    return attention(q, k, v, mod="temp", head_param=temps, mask=CAUSAL, scale=scale,
                     cu_seqlens=cu_seqlens)


def sigmoid_attn(q, k, v, *, causal: bool = True, bias: float = 0.0,
                 scale: Optional[float] = None, cu_seqlens=None):
    """``sigmoid(s+bias)*mask @ v``, mask after the sigmoid (``sigmoid_fix.py:34-40``)."""
    return attention(q, k, v, norm="sigmoid", sig_bias=bias, mask=CAUSAL if causal else FULL,
                     scale=scale, cu_seqlens=cu_seqlens)


def relu_attn(q, k, v, *, causal: bool = True, out_scale: float = 1.0,
              scale: Optional[float] = None, cu_seqlens=None):
    """``relu(s)*mask @ v * out_scale`` (``extra_bench.py:44``)."""
    return attention(q, k, v, norm="relu", out_scale=out_scale,
                     mask=CAUSAL if causal else FULL, scale=scale, cu_seqlens=cu_seqlens)


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


def op_config(op: str, **kw) -> Mask:
    """Mask of reference operator ``op`` with the given keyword overrides."""
    if op in ("softcap_gemma2", "sigmoid_attn", "relu_attn"):
        return CAUSAL if kw.get("causal", True) else FULL
    if op in ("bias_alibi", "temp_perhead"):
        return CAUSAL
    if op == "bias_sliding_window":
        w = kw.get("window", 256)
        return Mask(left=w - 1, right=0)
    if op == "bias_local":
        w = kw.get("window", 256)
        return Mask(left=w - 1, right=w - 1)
    if op == "bias_block_diagonal":
        return Mask(left=-1, right=0 if kw.get("causal", True) else -1,
                    block=kw.get("block", 512))
    if op == "bias_dilated":
        return Mask(left=-1, right=0, dilation=kw.get("dilation", 4))
    if op == "bias_prefix_lm":
        return Mask(left=-1, right=0, prefix=kw.get("prefix", 256))
    raise KeyError(op)


def visible_pairs(mask: Mask, seqlen_q: int, seqlen_kv: Optional[int] = None) -> int:
    """Visible (i, j) pairs of ``mask`` for one (batch, head) (host-side, no GPU)."""
    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.seqlen_q = seqlen_q
    p.seqlen_kv = seqlen_q if seqlen_kv is None else seqlen_kv
    p.win_left, p.win_right = mask.left, mask.right
    p.block, p.prefix, p.dilation = mask.block, mask.prefix, mask.dilation
    n = N.load().chia_attn_visible_pairs(ctypes.byref(p))
    if n < 0:
        raise ValueError(f"invalid mask {mask}")
    return int(n)


def tile_plan(mask: Mask, seqlen_q: int, row0: int, tile_m: int = 128, tile_n: int = 128,
              seqlen_kv: Optional[int] = None):
    """Key tiles ``(lo, hi, full_bits)`` the kernel visits for query rows ``[row0, row0+tile_m)``."""
    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.seqlen_q = seqlen_q
    p.seqlen_kv = seqlen_q if seqlen_kv is None else seqlen_kv
    p.win_left, p.win_right = mask.left, mask.right
    p.block, p.prefix, p.dilation = mask.block, mask.prefix, mask.dilation
    lo, hi, bits = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64()
    N.check(N.load().chia_attn_tile_plan(ctypes.byref(p), row0, tile_m, tile_n,
                                         ctypes.byref(lo), ctypes.byref(hi), ctypes.byref(bits)))
    return lo.value, hi.value, bits.value


def mask_aware_flops(mask: Mask, B: int, H: int, S: int, D: int) -> int:
    """``4 * D * visible_pairs * B * H`` -- the metric's FLOP count."""
    return 4 * D * visible_pairs(mask, S) * B * H
