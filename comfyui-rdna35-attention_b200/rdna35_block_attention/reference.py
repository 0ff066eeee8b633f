"""Public PyTorch reference helpers of the fixed-block API.

The reference exports these names from rdna35_block_attention/reference.py
(its test suite and nodes call them); the semantics kept are:

* layouts ``bhtd`` [B,H,T,D], ``bh_t_d`` [BH,T,D] and ``bthd`` [B,T,H*D]
  (with ``heads``), plus their aliases and ``auto`` (rank 4 -> bhtd, rank 3 ->
  bh_t_d); ``normalize_qkv_to_bh_t_d`` returns contiguous [BH,T,D] q/k/v and a
  ``LayoutInfo`` whose ``restore`` maps a [BH,T,D] result back;
* masks: [T,T] for every (batch, head); [N,T,T] with N = B (per batch, when
  the layout knows B and H), 1 or B*H; [B|1, H|1, T, T].  Boolean masks keep
  True entries, other masks are added to the scores;
* ``fixed_block_attention_ref``: FP32 softmax attention restricted to each
  64-token diagonal block (optionally causal, optionally masked);
  ``fixed_block_attention_sdpa`` the same through SDPA with a block mask;
  ``full_attention_sdpa_bhtd`` plain SDPA.

They are the explicit, opt-in reference modes (``mode="reference"``), never
a silent substitute for the B200 kernels.  This module expands a mask once
into a broadcastable [BH|1, T, T] view (``canonical_mask``), which the block
loop slices and the native masked kernel packs into bit words.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import torch

_LAYOUT_ALIASES = {
    "auto": "auto", "bhtd": "bhtd", "b,h,t,d": "bhtd", "bh_t_d": "bh_t_d", "bhtd_flat": "bh_t_d",
    "bhtdflat": "bh_t_d", "bthd": "bthd", "b,t,h*d": "bthd", "b_t_hd": "bthd",
}


@dataclass(frozen=True)
class LayoutInfo:
    layout: str
    batch: int | None
    heads: int | None
    tokens: int
    head_dim: int
    restore: Callable[[torch.Tensor], torch.Tensor]


def canonical_layout(layout: str) -> str:
    key = layout.lower().replace("-", "_").replace(" ", "")
    try:
        return _LAYOUT_ALIASES[key]
    except KeyError:
        raise ValueError(f"Unsupported layout '{layout}'.") from None


def _flatten_bhtd(x: torch.Tensor, heads):
    if x.ndim != 4:
        raise ValueError(f"layout='bhtd' expects [B,H,T,D], got rank {x.ndim}.")
    b, h, t, d = x.shape
    return (lambda y: y.contiguous().reshape(b * h, t, d)), \
        LayoutInfo("bhtd", b, h, t, d, lambda out: out.reshape(b, h, t, d))


def _flatten_bh_t_d(x: torch.Tensor, heads):
    if x.ndim != 3:
        raise ValueError(f"layout='bh_t_d' expects [BH,T,D], got rank {x.ndim}.")
    bh, t, d = x.shape
    return (lambda y: y.contiguous()), LayoutInfo("bh_t_d", None, None, t, d, lambda out: out.reshape(bh, t, d))


def _flatten_bthd(x: torch.Tensor, heads):
    if x.ndim != 3:
        raise ValueError(f"layout='bthd' expects [B,T,H*D], got rank {x.ndim}.")
    if heads is None or heads <= 0:
        raise ValueError("layout='bthd' requires a positive heads argument.")
    b, t, channels = x.shape
    if channels % heads:
        raise ValueError(f"channels={channels} is not divisible by heads={heads}.")
    d = channels // heads

    def flatten(y):
        return y.contiguous().view(b, t, heads, d).transpose(1, 2).reshape(b * heads, t, d)

    def restore(out):
        return out.view(b, heads, t, d).transpose(1, 2).reshape(b, t, channels)

    return flatten, LayoutInfo("bthd", b, heads, t, d, restore)


_FLATTENERS = {"bhtd": _flatten_bhtd, "bh_t_d": _flatten_bh_t_d, "bthd": _flatten_bthd}


def normalize_qkv_to_bh_t_d(q, k, v, *, layout: str = "auto", heads: int | None = None):
    """(q, k, v) as contiguous [BH,T,D] plus the LayoutInfo that restores a
    [BH,T,D] result to the caller's layout."""
    if not (q.shape == k.shape == v.shape):
        raise ValueError(f"Fixed block self-attention requires q/k/v to have identical shapes, got {q.shape}, "
                         f"{k.shape}, {v.shape}.")
    chosen = canonical_layout(layout)
    if chosen == "auto":
        chosen = {4: "bhtd", 3: "bh_t_d"}.get(q.ndim)
        if chosen is None:
            raise ValueError(f"Cannot infer layout for rank-{q.ndim} tensor.")
    flatten, info = _FLATTENERS[chosen](q, heads)
    return flatten(q), flatten(k), flatten(v), info


def canonical_mask(mask: torch.Tensor, info: LayoutInfo, batch_heads: int) -> torch.Tensor:
    """The mask as a [BH, T, T] or [1, T, T] (broadcast) view, following the
    rank rules of the module docstring; raises ValueError for shapes that do
    not fit the call."""
    t = info.tokens
    if mask.ndim not in (2, 3, 4):
        raise ValueError(f"Unsupported mask rank {mask.ndim}.")
    if tuple(mask.shape[-2:]) != (t, t):
        raise ValueError(f"{mask.ndim}D mask must end with [T,T], got {tuple(mask.shape)}.")
    if mask.ndim == 2:
        return mask.unsqueeze(0)
    if mask.ndim == 3:
        n = mask.shape[0]
        if info.batch is not None and info.heads is not None and n == info.batch:
            return mask.repeat_interleave(info.heads, dim=0)
        if n in (1, batch_heads):
            return mask
        raise ValueError(f"3D mask batch dimension {n} is not compatible with BH={batch_heads}.")
    if info.batch is None or info.heads is None:
        raise ValueError("4D mask requires a layout with known B and H.")
    if mask.shape[0] not in (1, info.batch) or mask.shape[1] not in (1, info.heads):
        raise ValueError(f"4D mask shape {tuple(mask.shape)} is not compatible with B={info.batch}, H={info.heads}.")
    return mask.expand(info.batch, info.heads, t, t).reshape(batch_heads, t, t)


def _mask_block(mask, start, end, *, batch_heads, info: LayoutInfo, device):
    """The [start:end] diagonal block of `mask` for every (batch, head)."""
    if mask is None:
        return None
    full = canonical_mask(mask.to(device=device), info, batch_heads)
    return full[:, start:end, start:end].expand(batch_heads, end - start, end - start)


def _apply_mask(scores: torch.Tensor, block_mask: torch.Tensor | None) -> torch.Tensor:
    if block_mask is None:
        return scores
    if block_mask.dtype == torch.bool:
        return scores.masked_fill(~block_mask, -torch.inf)
    return scores + block_mask.to(scores.dtype)


def fixed_block_attention_ref(q, k, v, block_size: int = 64, scale: float | None = None, causal: bool = False,
                              layout: str = "auto", *, heads: int | None = None, mask=None):
    """FP32 softmax attention inside each diagonal block of `block_size`
    tokens, result in the inputs' dtype and layout."""
    qf, kf, vf, info = normalize_qkv_to_bh_t_d(q, k, v, layout=layout, heads=heads)
    if block_size <= 0:
        raise ValueError("block_size must be positive.")
    bh, t, d = qf.shape
    scale_value = 1.0 / math.sqrt(d) if scale is None else float(scale)
    out = torch.empty_like(qf)
    for start in range(0, t, block_size):
        end = min(t, start + block_size)
        scores = (qf[:, start:end].float() @ kf[:, start:end].float().transpose(-2, -1)) * scale_value
        if causal:
            upper = torch.ones((end - start, end - start), dtype=torch.bool, device=q.device).triu(1)
            scores = scores.masked_fill(upper, -torch.inf)
        scores = _apply_mask(scores, _mask_block(mask, start, end, batch_heads=bh, info=info, device=q.device))
        out[:, start:end] = (torch.softmax(scores, dim=-1) @ vf[:, start:end].float()).to(qf.dtype)
    return info.restore(out)


def fixed_block_attention_bthd(q, k, v, heads: int, block_size: int = 64, scale: float | None = None,
                               causal: bool = False, *, mask=None):
    return fixed_block_attention_ref(q, k, v, block_size=block_size, scale=scale, causal=causal, layout="bthd",
                                     heads=heads, mask=mask)


def block_diagonal_sdpa_mask(tokens: int, *, block_size: int = 64, causal: bool = False, device=None):
    """[T,T] boolean mask: True where query and key share a block (and, when
    causal, the key is not after the query)."""
    if block_size <= 0:
        raise ValueError("block_size must be positive.")
    block = torch.arange(tokens, device=device) // block_size
    allowed = block[:, None] == block[None, :]
    if causal:
        allowed &= torch.ones((tokens, tokens), dtype=torch.bool, device=device).tril()
    return allowed


def fixed_block_attention_sdpa(q, k, v, block_size: int = 64, scale: float | None = None, causal: bool = False,
                               layout: str = "auto", *, heads: int | None = None):
    qf, kf, vf, info = normalize_qkv_to_bh_t_d(q, k, v, layout=layout, heads=heads)
    allowed = block_diagonal_sdpa_mask(info.tokens, block_size=block_size, causal=causal, device=qf.device)
    extra = {} if scale is None else {"scale": float(scale)}
    out = torch.nn.functional.scaled_dot_product_attention(qf.unsqueeze(1), kf.unsqueeze(1), vf.unsqueeze(1),
                                                           attn_mask=allowed, **extra)
    return info.restore(out.squeeze(1).to(qf.dtype))


def full_attention_sdpa_bhtd(q, k, v, *, scale: float | None = None, causal: bool = False):
    extra = {} if scale is None else {"scale": float(scale)}
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal, **extra)
