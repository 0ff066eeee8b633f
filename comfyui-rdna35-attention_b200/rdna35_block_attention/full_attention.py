"""Exact full online-softmax attention on B200 (mirrors the reference's
rdna35_block_attention/full_attention.py:25-103 contract: validation with
reason strings, ValueError when unsupported, optional diagnostics).  The
kernel is the tcgen05/TMEM attention of libb200attn.so (TMA-staged tiles,
two softmax warpgroups); D=64 inputs use its warp-MMA variant."""
from __future__ import annotations

import math
from typing import Any

import torch

from . import device

SUPPORTED_HEAD_DIMS = {64, 128}
SUPPORTED_DTYPES = {torch.float16, torch.bfloat16}


def _kernel_config(head_dim: int) -> dict[str, Any]:
    if head_dim == 128:
        return {"kernel": "tcgen05", "block_m": 128, "block_n": 64, "kv_stages": 6, "softmax_warpgroups": 2}
    return {"kernel": "mma_sync", "block_m": 64, "block_n": 64}


def validate_full_attention_b200_bh(q, k, v) -> dict[str, Any]:
    reason = None
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        reason = "expected_rank_3_bh_q_or_k_d"
    elif q.shape[0] != k.shape[0] or k.shape[0] != v.shape[0]:
        reason = "batch_heads_mismatch"
    elif q.shape[2] != k.shape[2] or k.shape[2] != v.shape[2]:
        reason = "head_dim_mismatch"
    elif k.shape[1] != v.shape[1]:
        reason = "key_value_length_mismatch"
    elif q.shape[1] == 0 or k.shape[1] == 0:
        reason = "empty_sequence"
    elif q.dtype != k.dtype or k.dtype != v.dtype:
        reason = "qkv_dtype_mismatch"
    elif q.dtype not in SUPPORTED_DTYPES:
        reason = f"unsupported_dtype_{q.dtype}"
    elif q.shape[2] not in SUPPORTED_HEAD_DIMS:
        reason = f"unsupported_head_dim_{q.shape[2]}"
    elif q.device != k.device or k.device != v.device:
        reason = "qkv_device_mismatch"
    elif q.device.type != "cuda":
        reason = f"not_cuda_device_{q.device.type}"
    elif not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
        reason = "qkv_must_be_contiguous"
    elif any(t.requires_grad for t in (q, k, v)):
        reason = "forward_only_requires_grad_not_supported"
    else:
        index, why = device.b200_device_index()
        if index is None:
            reason = "sm100_device_not_detected"
    head_dim = q.shape[2] if q.ndim == 3 else None
    return {
        "supported": reason is None,
        "reason": reason,
        "backend": "b200" if reason is None else None,
        "exact": True,
        "causal": False,
        "mask": None,
        "layout": "bhqd",
        "batch_heads": q.shape[0] if q.ndim == 3 else None,
        "q_tokens": q.shape[1] if q.ndim == 3 else None,
        "kv_tokens": k.shape[1] if k.ndim == 3 else None,
        "head_dim": head_dim,
        "dtype": str(q.dtype),
        "device": str(q.device),
        "config": _kernel_config(head_dim) if head_dim in SUPPORTED_HEAD_DIMS else None,
    }


def full_attention_b200(q, k, v, *, scale: float | None = None, return_diagnostics: bool = False):
    info = validate_full_attention_b200_bh(q, k, v)
    if not info["supported"]:
        raise ValueError(f"Full attention B200 path is unavailable: {info['reason']}")
    native = device.native_module()
    scale_value = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[2])
    out = native.full_attention(q, k, v, scale_value)
    return (out, info) if return_diagnostics else out


# the reference's public name for this entry point
full_attention_triton = full_attention_b200
validate_full_attention_triton_bh = validate_full_attention_b200_bh
