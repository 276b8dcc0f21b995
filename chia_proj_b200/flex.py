"""A ``flex_attention``-compatible frontend.

The reference benchmarks eight of its ten operators through PyTorch's
``flex_attention`` as ``score_mod`` / ``mask_mod`` callables
(JoshiP-commits/CHIA_proj ``extra_bench.py:85-99``; called as
``flex_attention(q, k, v, score_mod=..., block_mask=create_block_mask(...))``
at ``extra_bench.py:130-137``). This module accepts the same callables with
the same call signatures and runs them on the library's sm_100a kernels:

* ``create_block_mask(mask_mod, B, H, Q_LEN, KV_LEN, device=...)``
  evaluates ``mask_mod`` on the index grid and fits it to the library's mask
  model (``Mask``: window left / right, block, prefix, dilation), checking
  the fit element by element on the evaluated grid;
* ``flex_attention(query, key, value, score_mod=None, block_mask=None,
  scale=None, enable_gqa=False, return_lse=False)`` identifies ``score_mod``
  by evaluating it on probe scores and indices: identity, a per-head
  multiplier (temperature), an additive per-head slope times ``kv - q``
  (ALiBi) or ``cap * tanh(s / cap)`` (softcap).

Callables that fit none of these (a mask that depends on the batch or head,
a score_mod mixing two modifications, ...) raise ``NotExpressible``; like
the reference (``extra_bench.py:96-99``), sigmoid and ReLU attention are not
expressible here, because flex normalises with softmax -- they have their
own operators.

Evaluation happens once per block mask and once per (score_mod, heads,
device); callables must be written with broadcasting torch operations, as
flex requires.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, Optional, Tuple

import torch

from .ops import Mask, attention

__all__ = ["NotExpressible", "BlockMask", "create_block_mask", "flex_attention",
           "fit_mask", "identify_score_mod"]

# Largest number of (query, key) entries evaluated densely; larger masks are
# evaluated on a sample of rows (all of the first and last rows, and a stride).
DENSE_LIMIT = 1 << 24


class NotExpressible(ValueError):
    """The callable has no exact counterpart in the library's kernels."""


# ---------------------------------------------------------------- masks
def _mask_dense(m: Mask, rows: torch.Tensor, kv_len: int) -> torch.Tensor:
    """The visibility rule of ``Mask`` (``include/chia_attn.h``) on rows x keys."""
    i = rows.view(-1, 1)
    j = torch.arange(kv_len, device=rows.device).view(1, -1)
    band = torch.ones(i.shape[0], kv_len, dtype=torch.bool, device=rows.device)
    if m.left >= 0:
        band &= (i - j) <= m.left
    if m.right >= 0:
        band &= (j - i) <= m.right
    if m.block > 0:
        band &= torch.div(i, m.block, rounding_mode="floor") == \
            torch.div(j, m.block, rounding_mode="floor")
    if m.dilation > 1:
        band &= torch.remainder(i - j, m.dilation) == 0
    return band | (j < m.prefix)


def _sample_rows(q_len: int, kv_len: int) -> torch.Tensor:
    if q_len * kv_len <= DENSE_LIMIT:
        return torch.arange(q_len)
    n = max(64, DENSE_LIMIT // kv_len)
    head = torch.arange(min(q_len, n // 4))
    tail = torch.arange(max(0, q_len - n // 4), q_len)
    mid = torch.linspace(0, q_len - 1, n // 2).round().long()
    return torch.unique(torch.cat([head, tail, mid]))


def fit_mask(vis: torch.Tensor, rows: torch.Tensor, kv_len: int) -> Mask:
    """The simplest ``Mask`` whose visibility equals ``vis`` (rows x keys, for
    the query indices ``rows``) exactly; raises ``NotExpressible``."""
    vis = vis.to(torch.bool).cpu()
    rows = rows.cpu()
    n_rows = vis.shape[0]
    # an always-visible prefix: the leading keys every row sees
    full_cols = vis.all(0)
    p_max = int(full_cols.long().cumprod(0).sum().item()) if n_rows else 0
    j = torch.arange(kv_len)
    for prefix in ([0, p_max] if p_max else [0]):
        v2 = vis.clone()
        v2[:, :prefix] = False
        has = v2.any(1)
        if not has.any():
            cand = [Mask(left=-1, right=-1, prefix=prefix)] if prefix else []
        else:
            r = rows[has]
            lo = torch.where(v2[has], j.view(1, -1), kv_len).min(1).values
            hi = torch.where(v2[has], j.view(1, -1), -1).max(1).values
            # dilation: gcd of the gaps between consecutive visible keys of a row
            nz = v2[has].nonzero()
            same_row = nz[1:, 0] == nz[:-1, 0]
            gaps = torch.unique((nz[1:, 1] - nz[:-1, 1])[same_row]).tolist()
            dil = 0
            for gap in gaps:
                dil = math.gcd(dil, int(gap))
            dil = max(dil, 1)
            left_opts = [-1]
            lmax = int((r - lo).max().item())
            if lmax >= 0:
                left_opts.append(lmax)
            right_opts = [-1]
            rmax = int((hi - r).max().item())
            if rmax >= 0:
                right_opts.append(rmax)
            block_opts = [0]
            starts = (lo == r) & (r > 0)
            if starts.any():
                bsz = int(r[starts].min().item())
                if bsz > 0:
                    block_opts.append(bsz)
            cand = [Mask(left=lft, right=rgt, block=blk, prefix=prefix, dilation=dil)
                    for blk in block_opts for lft in left_opts for rgt in right_opts]
        for m in cand:
            try:
                m.validate()
            except ValueError:
                continue
            if torch.equal(_mask_dense(m, rows, kv_len), vis):
                return m
    raise NotExpressible("mask_mod matches no window / block / prefix / dilation mask "
                         "of the library")


@dataclass
class BlockMask:
    """Result of ``create_block_mask``: the fitted mask and the shape it was
    made for (the counterpart of flex's ``BlockMask``)."""

    mask: Mask
    q_len: int
    kv_len: int
    BLOCK_SIZE: Tuple[int, int] = (128, 128)

    @property
    def shape(self):
        return (self.q_len, self.kv_len)


def create_block_mask(mask_mod: Callable, B: Optional[int], H: Optional[int], Q_LEN: int,
                      KV_LEN: int, device="cuda", BLOCK_SIZE=128, _compile=False) -> BlockMask:
    """Same signature as ``torch.nn.attention.flex_attention.create_block_mask``.

    ``mask_mod(b, h, q_idx, kv_idx) -> bool tensor`` is evaluated on the index
    grid (on ``device``, so callables that capture device tensors work) for
    batch and head 0, and for the last batch and head when ``B`` / ``H`` are
    given (a mask that differs between them is not expressible)."""
    rows = _sample_rows(Q_LEN, KV_LEN)
    dev = torch.device(device) if not isinstance(device, torch.device) else device
    if dev.type == "cuda" and not torch.cuda.is_available():
        dev = torch.device("cpu")
    qi = rows.to(dev).view(-1, 1)
    kj = torch.arange(KV_LEN, device=dev).view(1, -1)

    def ev(b, h):
        z = torch.zeros((), dtype=torch.long, device=dev)
        out = mask_mod(z + b, z + h, qi, kj)
        return torch.broadcast_to(torch.as_tensor(out, device=dev), (qi.shape[0], KV_LEN))

    vis = ev(0, 0)
    for b, h in (((B or 1) - 1, 0), (0, (H or 1) - 1)):
        if (b, h) != (0, 0) and not torch.equal(ev(b, h), vis):
            raise NotExpressible("mask_mod depends on the batch or head index")
    bs = (BLOCK_SIZE, BLOCK_SIZE) if isinstance(BLOCK_SIZE, int) else tuple(BLOCK_SIZE)
    return BlockMask(fit_mask(vis, rows, KV_LEN), Q_LEN, KV_LEN, bs)


# ------------------------------------------------------------ score mods
@dataclass(frozen=True)
class ScoreMod:
    """An identified score_mod: ``mod`` of ``attention()`` and its parameters."""

    mod: str                                # none, temp, alibi, softcap
    head_param: Optional[torch.Tensor] = None  # [H] temperatures or slopes
    softcap: float = 30.0


def identify_score_mod(score_mod: Optional[Callable], H: int, device) -> ScoreMod:
    """Identify ``score_mod(score, b, h, q_idx, kv_idx)`` by evaluating it."""
    if score_mod is None:
        return ScoreMod("none")
    dev = torch.device(device)
    xs = torch.tensor([-7.0, -1.5, -0.25, 0.0, 0.5, 2.0, 9.0], device=dev)
    pos = [(0, 0), (5, 2), (3, 11), (40, 17), (100, 100)]
    X = xs.view(-1, 1, 1).expand(-1, H, len(pos))
    hh = torch.arange(H, device=dev).view(1, -1, 1).expand_as(X)
    qi = torch.tensor([p[0] for p in pos], device=dev).view(1, 1, -1).expand_as(X)
    kj = torch.tensor([p[1] for p in pos], device=dev).view(1, 1, -1).expand_as(X)
    b = torch.zeros_like(hh)
    with torch.no_grad():
        F = torch.as_tensor(score_mod(X.clone(), b, hh, qi, kj), device=dev).float()
        F = torch.broadcast_to(F, X.shape)
    Xf = X.float()
    tol = lambda a, c: bool(torch.allclose(a, c, rtol=1e-4, atol=1e-4))
    if tol(F, Xf):
        return ScoreMod("none")
    # temperature: F = t_h * s, t_h independent of the position
    t = F[xs.tolist().index(2.0)] / 2.0  # [H, P]
    th = t[:, 0]
    if tol(F, Xf * th.view(1, -1, 1)) and tol(t, th.view(-1, 1).expand_as(t)):
        return ScoreMod("temp", head_param=th.detach().float().cpu())
    # ALiBi: F = s + slope_h * (kv - q)
    d = F - Xf
    rel = (kj - qi).float()
    nz = rel[0, 0] != 0
    if nz.any():
        slope = (d[0][:, nz] / rel[0][:, nz])[:, 0]
        if tol(d, slope.view(1, -1, 1) * rel):
            return ScoreMod("alibi", head_param=slope.detach().float().cpu())
    # softcap: F = c tanh(s / c), c the saturation value
    big = torch.full((1, 1, 1, 1), 1e6, device=dev)
    z = torch.zeros((1, 1, 1, 1), dtype=torch.long, device=dev)
    with torch.no_grad():
        c = float(torch.as_tensor(score_mod(big.clone().squeeze(0), z[0], z[0], z[0], z[0]),
                                  device=dev).float().reshape(-1)[0])
    if math.isfinite(c) and c > 0 and tol(F, c * torch.tanh(Xf / c)):
        return ScoreMod("softcap", softcap=c)
    raise NotExpressible("score_mod is not the identity, a per-head temperature, "
                         "an ALiBi slope or a tanh softcap")


_score_cache: Dict[tuple, ScoreMod] = {}


def flex_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   score_mod: Optional[Callable] = None, block_mask: Optional[BlockMask] = None,
                   scale: Optional[float] = None, enable_gqa: bool = False,
                   return_lse: bool = False, kernel_options=None):
    """Same call as ``torch.nn.attention.flex_attention.flex_attention``, run
    on the library's kernels. ``block_mask=None`` means every key is visible
    (flex's default). Returns ``out`` or ``(out, lse)`` with the natural
    log-sum-exp when ``return_lse``."""
    B, H, Sq, D = query.shape
    Hkv, Skv = key.shape[1], key.shape[2]
    if Hkv != H and not enable_gqa:
        raise ValueError("query and key head counts differ: pass enable_gqa=True")
    if block_mask is None:
        mask = Mask(left=-1, right=-1)
    else:
        if block_mask.q_len != Sq or block_mask.kv_len != Skv:
            raise ValueError(f"block_mask was made for {block_mask.shape}, "
                             f"inputs are {(Sq, Skv)}")
        mask = block_mask.mask
    key_ = (id(score_mod), H, str(query.device))
    sm = _score_cache.get(key_) if score_mod is not None else ScoreMod("none")
    if sm is None:
        sm = identify_score_mod(score_mod, H, query.device)
        _score_cache[key_] = sm
    kw = {}
    if sm.mod == "softcap":
        kw["softcap"] = sm.softcap
    if sm.mod in ("temp", "alibi"):
        kw["head_param"] = sm.head_param
    return attention(query, key, value, mod=sm.mod, mask=mask, scale=scale,
                     return_lse=return_lse, **kw)
