"""ComfyUI model-local override for fixed block-diagonal attention (mirrors
the reference's rdna35_block_attention/comfy_patch.py:48-203: marker-gated
``exact_only`` / ``experimental_force_block_local`` modes, chaining to the
previous override or the original attention for every other call)."""
from __future__ import annotations

import logging
from typing import Any, Callable

from .dispatch import fixed_block_attention

LOG_PREFIX = "RDNA35 FixedBlockAttention (B200)"


def _fallback_call(previous_override: Callable | None, original_func: Callable, *args, **kwargs):
    if previous_override is not None:
        return previous_override(original_func, *args, **kwargs)
    return original_func(*args, **kwargs)


def _has_fixed_block_marker(kwargs: dict[str, Any]) -> bool:
    options = kwargs.get("transformer_options") or {}
    return "fixed_block_diagonal" in (kwargs.get("rdna35_attention_semantics"), options.get("rdna35_attention_semantics"))


def _declares_self_attention(q, k, v, kwargs: dict[str, Any]) -> bool:
    options = kwargs.get("transformer_options") or {}
    if kwargs.get("rdna35_is_self_attention") is True or options.get("rdna35_is_self_attention") is True:
        return True
    try:
        return q.data_ptr() == k.data_ptr() == v.data_ptr()
    except Exception:
        return False


def make_attention_override(*, mode: str, semantic_mode: str, block_size: int, causal: bool, verbose_fallbacks: bool,
                            previous_override: Callable | None) -> Callable:
    def attention_override(original_func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                           skip_output_reshape=False, **kwargs):
        call = dict(mask=mask, attn_precision=attn_precision, skip_reshape=skip_reshape,
                    skip_output_reshape=skip_output_reshape, **kwargs)
        eligible = _has_fixed_block_marker(kwargs)
        if not eligible and semantic_mode == "experimental_force_block_local":
            eligible = _declares_self_attention(q, k, v, kwargs)
        if not eligible:
            if verbose_fallbacks:
                logging.info("%s: original attention used; call is not proven fixed block-diagonal self-attention.",
                             LOG_PREFIX)
            return _fallback_call(previous_override, original_func, q, k, v, heads, **call)
        try:
            if skip_reshape:
                out, info = fixed_block_attention(q, k, v, block_size=block_size, causal=causal, layout="bhtd",
                                                  mode=mode, return_diagnostics=True, mask=mask)
                if not skip_output_reshape:
                    b, h, t, d = out.shape
                    out = out.transpose(1, 2).contiguous().reshape(b, t, h * d)
            else:
                out, info = fixed_block_attention(q, k, v, block_size=block_size, causal=causal, layout="bthd",
                                                  heads=heads, mode=mode, return_diagnostics=True, mask=mask)
                if skip_output_reshape:
                    b, t, c = out.shape
                    out = out.reshape(b, t, heads, c // heads).permute(0, 2, 1, 3).contiguous()
            if verbose_fallbacks and info.get("fallback_reason"):
                logging.info("%s: %s: %s", LOG_PREFIX, info.get("backend"), info.get("fallback_reason"))
            return out
        except Exception as exc:
            logging.warning("%s: fixed block attention failed; original attention used: %s: %s", LOG_PREFIX,
                            type(exc).__name__, exc)
            return _fallback_call(previous_override, original_func, q, k, v, heads, **call)

    return attention_override


def patch_model_attention(model, *, enabled: bool, mode: str, semantic_mode: str, block_size: int, causal: bool,
                          verbose_fallbacks: bool):
    if not enabled:
        return model, "disabled; model returned unchanged"
    if block_size != 64:
        return model, f"unsupported block_size={block_size}; only 64 is implemented, model returned unchanged"
    if semantic_mode not in {"exact_only", "experimental_force_block_local"}:
        return model, f"unsupported semantic_mode={semantic_mode}; model returned unchanged"
    if not hasattr(model, "clone") or not hasattr(model, "model_options"):
        return model, "MODEL does not expose ComfyUI ModelPatcher clone/model_options; model returned unchanged"
    clone = model.clone()
    options = clone.model_options.setdefault("transformer_options", {})
    previous = options.get("optimized_attention_override")
    options["optimized_attention_override"] = make_attention_override(
        mode=mode, semantic_mode=semantic_mode, block_size=block_size, causal=causal,
        verbose_fallbacks=verbose_fallbacks, previous_override=previous)
    if semantic_mode == "exact_only":
        info = ("model-local optimized_attention_override installed in exact_only mode; normal ComfyUI attention "
                "calls are left unchanged unless they explicitly declare "
                "rdna35_attention_semantics='fixed_block_diagonal'")
    else:
        info = ("model-local optimized_attention_override installed in experimental_force_block_local mode; only "
                "calls explicitly marked as fixed block-diagonal or self-attention are eligible; unproven calls "
                "fall back to the original attention backend")
    if previous is not None:
        info += "; existing optimized_attention_override is chained for fallback"
    return clone, info
