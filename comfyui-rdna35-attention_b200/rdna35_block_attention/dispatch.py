"""Fixed 64-token block-diagonal attention dispatch (mirrors the contract of
the reference's rdna35_block_attention/dispatch.py:82-186: same arguments,
``mode`` values, diagnostics dict and reason strings).

Eligible calls run the B200 kernel of libb200attn.so directly on the caller's
layout (BHTD, [BH,T,D] or BTHD viewed as BHTD, no copies).  Boolean and
float masks ([T,T], [N,T,T], [B|1,H|1,T,T]) run natively too: their
diagonal 64x64 blocks are packed on the device into FP32 score terms.
Requests the kernels do not implement -- masks of other dtypes, other block
sizes, tensors that require grad, CPU tensors -- use the PyTorch
reference; on an eligible CUDA call the native library must
be present (its absence raises instead of silently falling back)."""
from __future__ import annotations

from typing import Any

import torch

from . import device
from .reference import LayoutInfo, canonical_layout, canonical_mask, fixed_block_attention_ref

SUPPORTED_HEAD_DIMS = {32, 64, 128}
SUPPORTED_DTYPES = {torch.float16, torch.bfloat16, torch.float32}
NATIVE_MODES = {"b200", "triton"}  # "triton" kept as the reference's name for the optimized kernel


def _fallback(q, k, v, *, block_size, scale, causal, layout, heads, mask, reason, return_diagnostics):
    out = fixed_block_attention_ref(q, k, v, block_size=block_size, scale=scale, causal=causal, layout=layout,
                                    heads=heads, mask=mask)
    info = {"backend": "reference", "fallback_reason": reason, "optimized": False}
    return (out, info) if return_diagnostics else out


def _layout_of(q, k, v, layout: str, heads: int | None) -> tuple[str, int]:
    """Resolved layout name and head dimension, without copying anything."""
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"Fixed block self-attention requires q/k/v to have identical shapes, got {q.shape}, {k.shape}, {v.shape}.")
    chosen = canonical_layout(layout)
    if chosen == "auto":
        chosen = {4: "bhtd", 3: "bh_t_d"}.get(q.ndim)
        if chosen is None:
            raise ValueError(f"Cannot infer layout for rank-{q.ndim} tensor.")
    if chosen == "bhtd" and q.ndim == 4:
        return chosen, q.shape[-1]
    if chosen == "bh_t_d" and q.ndim == 3:
        return chosen, q.shape[-1]
    if chosen == "bthd" and q.ndim == 3:
        if heads is None or heads <= 0 or q.shape[-1] % heads:
            raise ValueError("layout='bthd' requires a positive heads argument dividing the channels.")
        return chosen, q.shape[-1] // heads
    raise ValueError(f"layout='{chosen}' does not match a rank-{q.ndim} tensor.")


NATIVE_MASK_DTYPES = {torch.bool, torch.float32, torch.float16, torch.bfloat16}


def _reject_reason(q_flat, k_flat, v_flat, head_dim, *, block_size, mask) -> str | None:
    if mask is not None and (not isinstance(mask, torch.Tensor) or mask.dtype not in NATIVE_MASK_DTYPES):
        return "arbitrary_mask_uses_reference"
    if any(t.requires_grad for t in (q_flat, k_flat, v_flat)):
        return "requires_grad_uses_reference"
    if block_size != 64:
        return f"unsupported_block_size_{block_size}"
    if q_flat.shape != k_flat.shape or q_flat.shape != v_flat.shape:
        return "qkv_shape_mismatch"
    if q_flat.dtype not in SUPPORTED_DTYPES or k_flat.dtype != q_flat.dtype or v_flat.dtype != q_flat.dtype:
        return f"unsupported_dtype_{q_flat.dtype}"
    d = head_dim
    if q_flat.dtype == torch.float32 and d > 128:
        return f"unsupported_head_dim_{d}"
    if q_flat.dtype != torch.float32 and d not in SUPPORTED_HEAD_DIMS:
        return f"unsupported_head_dim_{d}"
    if q_flat.device != k_flat.device or q_flat.device != v_flat.device:
        return "qkv_device_mismatch"
    if q_flat.device.type != "cuda":
        return f"not_cuda_device_{q_flat.device.type}"
    index, reason = device.b200_device_index()
    if index is None:
        return "sm100_device_not_detected"
    return None


def _mask_bias(mask: torch.Tensor, q_bhtd: torch.Tensor, layout: str):
    """The mask's diagonal-block terms for the native kernels: the mask is
    read with the reference's rank rules (canonical_mask) as a [B*H|1,T,T]
    view and packed on the device."""
    batch, heads, tokens, dim = q_bhtd.shape
    known = layout != "bh_t_d"
    info = LayoutInfo(layout, batch if known else None, heads if known else None, tokens, dim, lambda out: out)
    full = canonical_mask(mask.to(device=q_bhtd.device), info, batch * heads)
    return device.native_module().block_mask_bias(full)


def _bhtd_view(x: torch.Tensor, layout: str, heads: int | None) -> torch.Tensor:
    if layout == "bhtd":
        return x
    if layout == "bh_t_d":
        return x.unsqueeze(1)
    b, t, c = x.shape
    return x.view(b, t, heads, c // heads).permute(0, 2, 1, 3)


def fixed_block_attention(q, k, v, *, block_size: int = 64, scale: float | None = None, causal: bool = False,
                          layout: str = "auto", heads: int | None = None, mode: str = "auto",
                          allow_approximate: bool = False, return_diagnostics: bool = False, mask=None) -> Any:
    del allow_approximate  # exact by construction
    if mode not in {"auto", "reference", "b200", "triton"}:
        raise ValueError("mode must be one of: auto, reference, b200 (alias: triton).")
    kwargs = dict(block_size=block_size, scale=scale, causal=causal, layout=layout, heads=heads, mask=mask,
                  return_diagnostics=return_diagnostics)
    if mode == "reference":
        return _fallback(q, k, v, reason="mode_reference", **kwargs)
    try:
        chosen, head_dim = _layout_of(q, k, v, layout, heads)
    except Exception as exc:  # layout errors are reported through the reference path
        return _fallback(q, k, v, reason=f"layout_normalization_failed_{type(exc).__name__}: {exc}", **kwargs)
    reason = _reject_reason(q, k, v, head_dim, block_size=block_size, mask=mask)
    if reason is not None:
        return _fallback(q, k, v, reason=reason if mode == "auto" else f"requested_b200_but_{reason}", **kwargs)
    native = device.native_module()
    import math

    scale_value = float(scale) if scale is not None else 1.0 / math.sqrt(head_dim)
    qv, kv, vv = (_bhtd_view(x, chosen, heads) for x in (q, k, v))
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    bias, bias_stride = None, 0
    try:
        if mask is not None:
            bias, bias_stride = _mask_bias(mask, qv, chosen)
        native.fixed_block_attention(qv, kv, vv, scale_value, causal, out=_bhtd_view(out, chosen, heads),
                                     mask_bias=bias, mask_bias_stride=bias_stride)
    except ValueError as exc:  # e.g. strides the 16-byte row kernels cannot address, or a mask shape
        return _fallback(q, k, v, reason=f"b200_rejected_{exc}", **kwargs)
    diag = {"backend": "b200", "fallback_reason": None, "optimized": True, "layout": chosen,
            "tokens": qv.shape[2], "head_dim": head_dim}
    return (out, diag) if return_diagnostics else out
