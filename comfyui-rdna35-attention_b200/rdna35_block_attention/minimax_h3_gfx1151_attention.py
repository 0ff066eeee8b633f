"""MiniMax-H3 interleaved-QKV attention override (mirrors the reference's
rdna35_block_attention/minimax_h3_gfx1151_attention.py:60-215: the same
eligibility ladder and reason strings, KV pack below 12000 tokens and QKV
pack above).

B200 behaviour: eligible calls run exact attention natively straight from
the interleaved [B,T,3,H,D] views (the TMA maps stride over the fused
projection, so no pack copy is needed) and write the merged [B,T,H*D]
output; ``pack_minimax_h3_qkv`` remains available and packs with the native
16-byte copy kernel when the chained backend must receive packed tensors
(``use_b200_attention=False``)."""
from __future__ import annotations

import logging
import math
from typing import Any, Callable

import torch

from . import device

LOG_PREFIX = "RDNA35 MiniMax-H3 (B200)"
MINIMAX_H3_HEADS = 56
MINIMAX_H3_HEAD_DIM = 128
MINIMAX_H3_MIN_PACK_TOKENS = 4608
MINIMAX_H3_PACK_ALL_TOKENS = 12000
MINIMAX_H3_MAX_PACK_TOKENS = 16500


def _fallback_call(previous_override: Callable | None, original_func: Callable, *args, **kwargs):
    if previous_override is not None:
        return previous_override(original_func, *args, **kwargs)
    return original_func(*args, **kwargs)


def _locate_minimax_h3(model: Any) -> Any | None:
    if hasattr(model, "get_model_object"):
        try:
            diffusion_model = model.get_model_object("diffusion_model")
        except (AttributeError, KeyError):
            diffusion_model = None
        if diffusion_model is not None:
            return diffusion_model
    return getattr(getattr(model, "model", None), "diffusion_model", None)


def _is_native_minimax_h3(model: Any) -> bool:
    dm = _locate_minimax_h3(model)
    return (dm is not None and type(dm).__module__ == "comfy.ldm.minimax.model"
            and type(dm).__name__ == "MiniMaxH3Model" and hasattr(dm, "blocks") and hasattr(dm, "hidden_size"))


def minimax_h3_pack_profile(tokens: int) -> str:
    return "qkv" if tokens >= MINIMAX_H3_PACK_ALL_TOKENS else "kv"


def pack_minimax_h3_qkv(q, k, v):
    """Pack K,V (T < 12000) or Q,K,V (T >= 12000) into one contiguous
    allocation; values are unchanged (minimax_h3_gfx1151_attention.py:64-74)."""
    profile = minimax_h3_pack_profile(q.shape[2])
    group = (q, k, v) if profile == "qkv" else (k, v)
    if q.is_cuda and q.stride(-1) == 1 and device.b200_device_index()[0] is not None:
        packed = device.native_module().pack_views(list(group))
    else:
        packed = torch.stack(group)
    if profile == "qkv":
        return packed[0], packed[1], packed[2], profile
    return q, packed[0], packed[1], profile


def minimax_h3_attention(q, k, v, *, scale: float | None = None):
    """Exact softmax attention of BHTD views (any token stride, e.g. the
    interleaved H3 projection) written as merged [B,T,H*D]."""
    b, h, t, d = q.shape
    out = torch.empty((b, t, h * d), device=q.device, dtype=q.dtype)
    scale_value = float(scale) if scale is not None else 1.0 / math.sqrt(d)
    device.native_module().full_attention(q, k, v, scale_value, out=out.view(b, t, h, d).transpose(1, 2))
    return out


def _reject_reason(q, k, v, heads, mask, skip_reshape, skip_output_reshape, device_index, kwargs) -> str | None:
    if mask is not None:
        return "attention_mask_is_not_supported"
    if not skip_reshape or skip_output_reshape:
        return "minimax_h3_merged_output_contract_is_required"
    if kwargs.get("enable_gqa", False):
        return "gqa_is_not_supported"
    if kwargs.get("is_causal", False) or kwargs.get("causal", False):
        return "causal_attention_is_not_supported"
    if kwargs.get("attn_bias") is not None:
        return "attention_bias_is_not_supported"
    if not all(isinstance(t, torch.Tensor) for t in (q, k, v)):
        return "qkv_are_not_tensors"
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        return "matching_bhtd_qkv_are_required"
    if q.shape[0] != 1 or q.shape[1] != MINIMAX_H3_HEADS or heads != MINIMAX_H3_HEADS or q.shape[3] != MINIMAX_H3_HEAD_DIM:
        return "minimax_h3_b1_h56_d128_is_required"
    if q.shape[2] < MINIMAX_H3_MIN_PACK_TOKENS:
        return f"tokens_below_{MINIMAX_H3_MIN_PACK_TOKENS}"
    if q.shape[2] > MINIMAX_H3_MAX_PACK_TOKENS:
        return f"tokens_above_{MINIMAX_H3_MAX_PACK_TOKENS}"
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        return "matching_bfloat16_qkv_are_required"
    if q.device != k.device or q.device != v.device or q.device.type != "cuda":
        return "matching_cuda_qkv_device_is_required"
    index = q.device.index if q.device.index is not None else torch.cuda.current_device()
    if index != device_index:
        return "qkv_are_not_on_the_validated_b200_device"
    if any(t.requires_grad for t in (q, k, v)):
        return "forward_only_requires_grad_not_supported"
    if any(t.stride(3) != 1 for t in (q, k, v)):
        return "contiguous_head_dimension_is_required"
    if q.is_contiguous() and k.is_contiguous() and v.is_contiguous():
        return "qkv_are_already_packed"
    return None


def make_minimax_h3_gfx1151_attention_override(*, device_index: int, verbose_fallbacks: bool,
                                               previous_override: Callable | None,
                                               use_b200_attention: bool = True) -> Callable:
    def attention_override(original_func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                           skip_output_reshape=False, **kwargs):
        call = dict(mask=mask, attn_precision=attn_precision, skip_reshape=skip_reshape,
                    skip_output_reshape=skip_output_reshape, **kwargs)
        reason = _reject_reason(q, k, v, heads, mask, skip_reshape, skip_output_reshape, device_index, kwargs)
        if reason is not None:
            if verbose_fallbacks:
                logging.info("%s: existing backend used: %s", LOG_PREFIX, reason)
            return _fallback_call(previous_override, original_func, q, k, v, heads, **call)
        if use_b200_attention:
            if verbose_fallbacks:
                logging.info("%s: native exact attention at T=%d", LOG_PREFIX, q.shape[2])
            return minimax_h3_attention(q, k, v, scale=kwargs.get("scale"))
        pq, pk, pv, profile = pack_minimax_h3_qkv(q, k, v)
        if verbose_fallbacks:
            logging.info("%s: packed %s at T=%d", LOG_PREFIX, profile.upper(), q.shape[2])
        return _fallback_call(previous_override, original_func, pq, pk, pv, heads, **call)

    return attention_override


make_minimax_h3_b200_attention_override = make_minimax_h3_gfx1151_attention_override


def patch_minimax_h3_gfx1151_attention(model, *, enabled: bool, verbose_fallbacks: bool,
                                       use_b200_attention: bool = True):
    if not enabled:
        return model, "disabled; model returned unchanged"
    if not hasattr(model, "clone") or not hasattr(model, "model_options"):
        return model, "MODEL does not expose ComfyUI ModelPatcher clone/model_options; model returned unchanged"
    if not _is_native_minimax_h3(model):
        return model, "native ComfyUI MiniMaxH3Model was not found; model returned unchanged"
    device_index, error = device.b200_device_index()
    if device_index is None:
        return model, f"{error}; model returned unchanged"
    previous = model.model_options.get("transformer_options", {}).get("optimized_attention_override")
    if previous is not None and getattr(previous, "container_function", None) is not None:
        return model, "container-aware optimized_attention_override is already installed; model returned unchanged"
    clone = model.clone()
    options = clone.model_options.setdefault("transformer_options", {})
    options["optimized_attention_override"] = make_minimax_h3_gfx1151_attention_override(
        device_index=device_index, verbose_fallbacks=verbose_fallbacks, previous_override=previous,
        use_b200_attention=use_b200_attention)
    info = (f"model-local MiniMax-H3 B200 override installed for BF16 B=1,H=56,D=128 with "
            f"{MINIMAX_H3_MIN_PACK_TOKENS}<=T<={MINIMAX_H3_MAX_PACK_TOKENS}; "
            + ("exact attention runs natively on the interleaved views" if use_b200_attention else
               f"KV is packed below T={MINIMAX_H3_PACK_ALL_TOKENS}, QKV at longer sequences, and the existing "
               "attention backend remains responsible for exact attention"))
    if previous is not None:
        info += "; existing optimized_attention_override is chained for fallback"
    return clone, info


patch_minimax_h3_b200_attention = patch_minimax_h3_gfx1151_attention
