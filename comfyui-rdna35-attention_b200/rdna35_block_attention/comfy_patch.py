"""ComfyUI model-local override for fixed 64-token block-diagonal attention.

Contract kept from the reference's rdna35_block_attention/comfy_patch.py:48-203
(names, keyword signatures, semantic modes, log and info strings are the
drop-in interface):

* ``make_attention_override(*, mode, semantic_mode, block_size, causal,
  verbose_fallbacks, previous_override)`` returns an override that runs
  fixed block-diagonal attention only on calls proven to have that meaning:
  calls carrying ``rdna35_attention_semantics='fixed_block_diagonal'`` (as a
  keyword or in ``transformer_options``) in both modes, and in
  ``experimental_force_block_local`` mode also calls that declare
  ``rdna35_is_self_attention=True`` or pass one tensor as q, k and v.  Every
  other call, and any call whose block attention raises, goes with all its
  arguments to the previous override or the original attention function.
  ComfyUI's two input layouts ([B,H,T,D] when ``skip_reshape``, else
  [B,T,H*D]) and two output layouts (``skip_output_reshape``) are honoured;
* ``patch_model_attention(model, ...)`` installs it on a clone and returns
  ``(model, info)``, or the unchanged model with the reason it was refused.

The eligibility rule per semantic mode is a table, and the input/output
layout handling is one small plan per ``skip_reshape`` value.
"""
from __future__ import annotations

import logging
from typing import Any, Callable

from .dispatch import fixed_block_attention

LOG_PREFIX = "RDNA35 FixedBlockAttention (B200)"
_MARKER = "fixed_block_diagonal"


def _fallback_call(previous_override: Callable | None, original_func: Callable, *args, **kwargs):
    if previous_override is None:
        return original_func(*args, **kwargs)
    return previous_override(original_func, *args, **kwargs)


def _option(kwargs: dict[str, Any], name: str) -> tuple[Any, Any]:
    """(keyword value, transformer_options value) of one call setting."""
    return kwargs.get(name), (kwargs.get("transformer_options") or {}).get(name)


def _has_fixed_block_marker(kwargs: dict[str, Any]) -> bool:
    return _MARKER in _option(kwargs, "rdna35_attention_semantics")


def _declares_self_attention(q, k, v, kwargs: dict[str, Any]) -> bool:
    if any(value is True for value in _option(kwargs, "rdna35_is_self_attention")):
        return True
    try:
        return q.data_ptr() == k.data_ptr() == v.data_ptr()
    except Exception:
        return False


# semantic mode -> is this call eligible for block-local attention?
_ELIGIBILITY: dict[str, Callable] = {
    "exact_only": lambda q, k, v, kwargs: _has_fixed_block_marker(kwargs),
    "experimental_force_block_local": lambda q, k, v, kwargs: (_has_fixed_block_marker(kwargs)
                                                               or _declares_self_attention(q, k, v, kwargs)),
}


def _block_attention(q, k, v, heads, skip_reshape, skip_output_reshape, **options):
    """Run the dispatcher in the caller's input layout and return the output
    in the layout ComfyUI asked for, with the dispatcher's diagnostics."""
    if skip_reshape:  # [B,H,T,D] in
        out, info = fixed_block_attention(q, k, v, layout="bhtd", return_diagnostics=True, **options)
        if not skip_output_reshape:
            batch, nh, tokens, dim = out.shape
            out = out.transpose(1, 2).contiguous().reshape(batch, tokens, nh * dim)
        return out, info
    out, info = fixed_block_attention(q, k, v, layout="bthd", heads=heads, return_diagnostics=True, **options)
    if skip_output_reshape:  # [B,T,H*D] -> [B,H,T,D]
        batch, tokens, width = out.shape
        out = out.reshape(batch, tokens, heads, width // heads).permute(0, 2, 1, 3).contiguous()
    return out, info


def make_attention_override(*, mode: str, semantic_mode: str, block_size: int, causal: bool, verbose_fallbacks: bool,
                            previous_override: Callable | None) -> Callable:
    eligible = _ELIGIBILITY.get(semantic_mode, _ELIGIBILITY["exact_only"])

    def attention_override(original_func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                           skip_output_reshape=False, **kwargs):
        def fall_back():
            return _fallback_call(previous_override, original_func, q, k, v, heads, mask=mask,
                                  attn_precision=attn_precision, skip_reshape=skip_reshape,
                                  skip_output_reshape=skip_output_reshape, **kwargs)

        if not eligible(q, k, v, kwargs):
            if verbose_fallbacks:
                logging.info("%s: original attention used; call is not proven fixed block-diagonal self-attention.",
                             LOG_PREFIX)
            return fall_back()
        try:
            out, info = _block_attention(q, k, v, heads, skip_reshape, skip_output_reshape, block_size=block_size,
                                         causal=causal, mode=mode, mask=mask)
        except Exception as exc:
            logging.warning("%s: fixed block attention failed; original attention used: %s: %s", LOG_PREFIX,
                            type(exc).__name__, exc)
            return fall_back()
        if verbose_fallbacks and info.get("fallback_reason"):
            logging.info("%s: %s: %s", LOG_PREFIX, info.get("backend"), info.get("fallback_reason"))
        return out

    return attention_override


_MODE_INFO = {
    "exact_only": ("model-local optimized_attention_override installed in exact_only mode; normal ComfyUI attention "
                   "calls are left unchanged unless they explicitly declare "
                   "rdna35_attention_semantics='fixed_block_diagonal'"),
    "experimental_force_block_local": ("model-local optimized_attention_override installed in "
                                       "experimental_force_block_local mode; only calls explicitly marked as fixed "
                                       "block-diagonal or self-attention are eligible; unproven calls fall back to "
                                       "the original attention backend"),
}


def patch_model_attention(model, *, enabled: bool, mode: str, semantic_mode: str, block_size: int, causal: bool,
                          verbose_fallbacks: bool):
    if not enabled:
        return model, "disabled; model returned unchanged"
    if block_size != 64:
        return model, f"unsupported block_size={block_size}; only 64 is implemented, model returned unchanged"
    if semantic_mode not in _MODE_INFO:
        return model, f"unsupported semantic_mode={semantic_mode}; model returned unchanged"
    if not (hasattr(model, "clone") and hasattr(model, "model_options")):
        return model, "MODEL does not expose ComfyUI ModelPatcher clone/model_options; model returned unchanged"
    clone = model.clone()
    options = clone.model_options.setdefault("transformer_options", {})
    previous = options.get("optimized_attention_override")
    options["optimized_attention_override"] = make_attention_override(
        mode=mode, semantic_mode=semantic_mode, block_size=block_size, causal=causal,
        verbose_fallbacks=verbose_fallbacks, previous_override=previous)
    info = _MODE_INFO[semantic_mode]
    if previous is not None:
        info += "; existing optimized_attention_override is chained for fallback"
    return clone, info
