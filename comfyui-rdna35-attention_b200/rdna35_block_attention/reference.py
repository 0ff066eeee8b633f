"""Public PyTorch reference helpers of the fixed-block API (the reference
exports them from rdna35_block_attention/reference.py): layout
normalisation to [BH,T,D], mask slicing, the block-diagonal loop, the SDPA
block-mask twin and full SDPA.  They are explicit, opt-in reference modes
(``mode="reference"``, arbitrary masks), never a silent substitute for the
B200 kernels."""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import torch

_LAYOUTS = {
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
    if key not in _LAYOUTS:
        raise ValueError(f"Unsupported layout '{layout}'.")
    return _LAYOUTS[key]


def normalize_qkv_to_bh_t_d(q, k, v, *, layout: str = "auto", heads: int | None = None):
    """(q, k, v) as contiguous [BH,T,D] plus LayoutInfo to restore the output
    (reference.py:38-111)."""
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"Fixed block self-attention requires q/k/v to have identical shapes, got {q.shape}, {k.shape}, {v.shape}.")
    chosen = canonical_layout(layout)
    if chosen == "auto":
        if q.ndim == 4:
            chosen = "bhtd"
        elif q.ndim == 3:
            chosen = "bh_t_d"
        else:
            raise ValueError(f"Cannot infer layout for rank-{q.ndim} tensor.")
    if chosen == "bhtd":
        if q.ndim != 4:
            raise ValueError(f"layout='bhtd' expects [B,H,T,D], got rank {q.ndim}.")
        b, h, t, d = q.shape
        flat = [x.contiguous().reshape(b * h, t, d) for x in (q, k, v)]
        return (*flat, LayoutInfo(chosen, b, h, t, d, lambda out: out.reshape(b, h, t, d)))
    if chosen == "bh_t_d":
        if q.ndim != 3:
            raise ValueError(f"layout='bh_t_d' expects [BH,T,D], got rank {q.ndim}.")
        bh, t, d = q.shape
        return (q.contiguous(), k.contiguous(), v.contiguous(),
                LayoutInfo(chosen, None, None, t, d, lambda out: out.reshape(bh, t, d)))
    if q.ndim != 3:
        raise ValueError(f"layout='bthd' expects [B,T,H*D], got rank {q.ndim}.")
    if heads is None or heads <= 0:
        raise ValueError("layout='bthd' requires a positive heads argument.")
    b, t, channels = q.shape
    if channels % heads != 0:
        raise ValueError(f"channels={channels} is not divisible by heads={heads}.")
    d = channels // heads

    def flatten(x):
        return x.contiguous().reshape(b, t, heads, d).permute(0, 2, 1, 3).contiguous().reshape(b * heads, t, d)

    def restore(out):
        return out.reshape(b, heads, t, d).permute(0, 2, 1, 3).contiguous().reshape(b, t, channels)

    return flatten(q), flatten(k), flatten(v), LayoutInfo(chosen, b, heads, t, d, restore)


def _mask_block(mask, start, end, *, batch_heads, info: LayoutInfo, device):
    """Slice the [start:end] diagonal block of a 2/3/4-D mask (reference.py:114-156)."""
    if mask is None:
        return None
    m = mask.to(device=device)
    t = info.tokens
    if m.shape[-2:] != (t, t):
        raise ValueError(f"{m.ndim}D mask must end with [T,T], got {tuple(m.shape)}.")
    if m.ndim == 2:
        return m[start:end, start:end].unsqueeze(0).expand(batch_heads, -1, -1)
    if m.ndim == 3:
        m = m[:, start:end, start:end]
        if info.batch is not None and m.shape[0] == info.batch and info.heads is not None:
            return m.repeat_interleave(info.heads, dim=0)
        if m.shape[0] == 1:
            return m.expand(batch_heads, -1, -1)
        if m.shape[0] == batch_heads:
            return m
        raise ValueError(f"3D mask batch dimension {m.shape[0]} is not compatible with BH={batch_heads}.")
    if m.ndim == 4:
        if info.batch is None or info.heads is None:
            raise ValueError("4D mask requires a layout with known B and H.")
        if m.shape[0] not in (1, info.batch) or m.shape[1] not in (1, info.heads):
            raise ValueError(f"4D mask shape {tuple(m.shape)} is not compatible with B={info.batch}, H={info.heads}.")
        m = m.expand(info.batch, info.heads, t, t)
        return m[:, :, start:end, start:end].reshape(batch_heads, end - start, end - start)
    raise ValueError(f"Unsupported mask rank {m.ndim}.")


def fixed_block_attention_ref(q, k, v, block_size: int = 64, scale: float | None = None, causal: bool = False,
                              layout: str = "auto", *, heads: int | None = None, mask=None):
    """Block-diagonal softmax attention loop in FP32 (reference.py:159-200)."""
    qf, kf, vf, info = normalize_qkv_to_bh_t_d(q, k, v, layout=layout, heads=heads)
    if block_size <= 0:
        raise ValueError("block_size must be positive.")
    bh, t, d = qf.shape
    scale_value = float(scale) if scale is not None else 1.0 / math.sqrt(d)
    out = torch.empty_like(qf)
    for start in range(0, t, block_size):
        end = min(start + block_size, t)
        scores = torch.matmul(qf[:, start:end].float(), kf[:, start:end].float().transpose(-2, -1)) * scale_value
        if causal:
            tri = torch.ones((end - start, end - start), dtype=torch.bool, device=q.device).triu(1)
            scores = scores.masked_fill(tri.unsqueeze(0), -torch.inf)
        block_mask = _mask_block(mask, start, end, batch_heads=bh, info=info, device=q.device)
        if block_mask is not None:
            scores = scores.masked_fill(~block_mask, -torch.inf) if block_mask.dtype == torch.bool else scores + block_mask.to(scores.dtype)
        out[:, start:end] = torch.matmul(torch.softmax(scores, dim=-1), vf[:, start:end].float()).to(qf.dtype)
    return info.restore(out)


def fixed_block_attention_bthd(q, k, v, heads: int, block_size: int = 64, scale: float | None = None,
                               causal: bool = False, *, mask=None):
    return fixed_block_attention_ref(q, k, v, block_size=block_size, scale=scale, causal=causal, layout="bthd",
                                     heads=heads, mask=mask)


def block_diagonal_sdpa_mask(tokens: int, *, block_size: int = 64, causal: bool = False, device=None):
    if block_size <= 0:
        raise ValueError("block_size must be positive.")
    pos = torch.arange(tokens, device=device)
    mask = (pos // block_size)[:, None] == (pos // block_size)[None, :]
    if causal:
        mask = mask & (pos[None, :] <= pos[:, None])
    return mask


def fixed_block_attention_sdpa(q, k, v, block_size: int = 64, scale: float | None = None, causal: bool = False,
                               layout: str = "auto", *, heads: int | None = None):
    qf, kf, vf, info = normalize_qkv_to_bh_t_d(q, k, v, layout=layout, heads=heads)
    mask = block_diagonal_sdpa_mask(info.tokens, block_size=block_size, causal=causal, device=qf.device)
    kwargs = {} if scale is None else {"scale": float(scale)}
    out = torch.nn.functional.scaled_dot_product_attention(qf[:, None], kf[:, None], vf[:, None], attn_mask=mask,
                                                           **kwargs).squeeze(1)
    return info.restore(out.to(qf.dtype))


def full_attention_sdpa_bhtd(q, k, v, *, scale: float | None = None, causal: bool = False):
    kwargs = {} if scale is None else {"scale": float(scale)}
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal, **kwargs)
