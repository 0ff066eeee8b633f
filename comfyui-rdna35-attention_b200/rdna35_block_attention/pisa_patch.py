"""PISA model patch and ``optimized_attention_override`` (mirrors the
reference's rdna35_block_attention/pisa_patch.py:41-284): the same reject
ladder and reason strings, chaining to the previous override, the Anima
direct ``attn_op`` install when the model validates, and the generic PISA
override otherwise.  The native backend is ``b200_pisa`` (sm_100a)."""
from __future__ import annotations

import importlib
import logging
import math
from typing import Any, Callable

import torch

from . import device
from .anima_pisa_integration import (ANIMA_PISA_FIRST_LAYER, ANIMA_PISA_LAST_LAYER, install_anima_pisa_attention,
                                     validate_anima_pisa_model)
from .generic_pisa import make_generic_pisa_override
from .pisa_runtime import PISA_RUNTIME_ATTACHMENT, PISARuntimeState

LOG_PREFIX = "RDNA35 PISA (B200)"
NATIVE_API = 7
TOKEN_POLICIES = {
    "anima_1536_spatial": frozenset((9216,)),
    "auto_9216": frozenset((9216,)),
}
SPATIAL_BLOCK_EDGE = 8
ANIMA_TOKEN_SHAPE = (1, 96, 96)


def _run_pisa_attention(native_forward: Callable, q, k, v, exact_budget: float, scale: float | None):
    total_blocks = math.ceil(q.shape[-2] / 64)
    exact_blocks = min(total_blocks, math.ceil(exact_budget * total_blocks))
    return native_forward(q, k, v, exact_blocks, scale=scale)


def _fallback_call(previous_override: Callable | None, original_func: Callable, *args, **kwargs):
    if previous_override is not None:
        return previous_override(original_func, *args, **kwargs)
    return original_func(*args, **kwargs)


def _device_index() -> tuple[int | None, str | None]:
    return device.b200_device_index()


def _pisa_reject_reason(q, k, v, heads, mask, attn_precision, skip_reshape, skip_output_reshape,
                        allowed_tokens: frozenset, expected_token_shape: tuple, device_index: int,
                        kwargs: dict[str, Any]) -> str | None:
    if kwargs.get("is_self_attention") is not True:
        return "call_is_not_explicitly_self_attention"
    if mask is not None:
        return "attention_mask_is_not_supported"
    if not skip_reshape:
        return "pre_reshaped_qkv_is_required"
    if skip_output_reshape:
        return "merged_attention_output_is_required"
    if not all(isinstance(t, torch.Tensor) for t in (q, k, v)):
        return "qkv_are_not_tensors"
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        return "matching_bhtd_qkv_are_required"
    if q.shape[0] <= 0 or q.shape[1] != heads or q.shape[-1] != 128:
        return "unsupported_batch_heads_or_head_dim"
    if q.shape[-2] not in allowed_tokens:
        return f"tokens_{q.shape[-2]}_are_not_enabled"
    token_shape = kwargs.get("attention_token_shape")
    if not isinstance(token_shape, (tuple, list)) or tuple(token_shape) != expected_token_shape:
        return f"token_shape_{token_shape}_is_not_{expected_token_shape}"
    side = math.isqrt(q.shape[-2])
    if side * side != q.shape[-2] or side % SPATIAL_BLOCK_EDGE:
        return "square_spatial_tokens_divisible_by_8_are_required"
    if kwargs.get("is_initial_transformer_block") is not False:
        return "initial_or_unmarked_transformer_block"
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        return "matching_bfloat16_qkv_are_required"
    if q.device != k.device or q.device != v.device:
        return "qkv_must_share_one_device"
    if q.device.type != "cuda":
        return "cuda_device_is_required"
    if q.device.index != device_index:
        return f"cuda_device_{q.device.index}_is_not_validated_device_{device_index}"
    expected_stride = (q.shape[1] * q.shape[2] * q.shape[3], q.shape[3], q.shape[1] * q.shape[3], 1)
    if any(t.stride() != expected_stride for t in (q, k, v)):
        return "bhtd_views_over_contiguous_bthd_storage_are_required"
    if any(t.requires_grad for t in (q, k, v)):
        return "forward_only_qkv_are_required"
    if attn_precision == torch.float32:
        return "float32_attention_precision_is_not_supported"
    if kwargs.get("enable_gqa", False):
        return "gqa_is_not_supported"
    return None


def make_pisa_attention_override(*, exact_budget: float, allowed_tokens: frozenset, expected_token_shape: tuple,
                                 device_index: int, native_forward: Callable, verbose_fallbacks: bool,
                                 previous_override: Callable | None) -> Callable:
    def attention_override(original_func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                           skip_output_reshape=False, **kwargs):
        reason = _pisa_reject_reason(q, k, v, heads, mask, attn_precision, skip_reshape, skip_output_reshape,
                                     allowed_tokens, expected_token_shape, device_index, kwargs)
        if reason is not None:
            if verbose_fallbacks:
                logging.info("%s: original attention used: %s", LOG_PREFIX, reason)
            return _fallback_call(previous_override, original_func, q, k, v, heads, mask=mask,
                                  attn_precision=attn_precision, skip_reshape=skip_reshape,
                                  skip_output_reshape=skip_output_reshape, **kwargs)
        return _run_pisa_attention(native_forward, q, k, v, exact_budget, kwargs.get("scale"))

    return attention_override


def patch_model_pisa_attention(model, *, enabled: bool, exact_budget: float, token_policy: str,
                               verbose_fallbacks: bool, start_layer: int = ANIMA_PISA_FIRST_LAYER,
                               end_layer: int = ANIMA_PISA_LAST_LAYER):
    if not enabled:
        return model, "disabled; model returned unchanged"
    if not 0.0 <= exact_budget <= 1.0:
        return model, f"invalid exact_budget={exact_budget}; model returned unchanged"
    if token_policy not in TOKEN_POLICIES:
        return model, f"unsupported token_policy={token_policy}; model returned unchanged"
    if not 0 <= start_layer <= end_layer < 28:
        return model, f"invalid Anima layer range {start_layer}:{end_layer}; model returned unchanged"
    if not hasattr(model, "clone") or not hasattr(model, "model_options"):
        return model, "MODEL does not expose ComfyUI ModelPatcher clone/model_options; model returned unchanged"
    device_index, device_error = _device_index()
    if device_index is None:
        return model, f"{device_error}; model returned unchanged"

    is_anima = False
    if hasattr(model, "get_model_object") and hasattr(model, "add_object_patch"):
        try:
            validate_anima_pisa_model(model)
            is_anima = True
        except (AttributeError, TypeError, ValueError):
            pass

    if not is_anima:
        clone = model.clone()
        state = PISARuntimeState(armed=True)
        if hasattr(clone, "set_attachments"):
            clone.set_attachments(PISA_RUNTIME_ATTACHMENT, state)
        options = clone.model_options.setdefault("transformer_options", {})
        previous = options.get("optimized_attention_override")
        options["optimized_attention_override"] = make_generic_pisa_override(
            exact_budget=exact_budget, device_index=device_index, previous_override=previous, runtime_state=state,
            validate_output=verbose_fallbacks)
        info = "model-local generic B200 PISA installed for explicit self-attention with T>=8192"
        if previous is not None:
            info += "; existing optimized_attention_override is chained for fallback"
        return clone, info

    try:
        native = importlib.import_module("b200_pisa")
        build_info = native.build_info()
        capabilities = native.capabilities()
        native.prepare()
    except (ImportError, OSError, RuntimeError, AttributeError) as exc:
        return model, f"b200_pisa is unavailable ({type(exc).__name__}: {exc}); model returned unchanged"
    if build_info.get("api") != NATIVE_API:
        return model, f"b200_pisa API {NATIVE_API} is required, got {build_info.get('api')}; model returned unchanged"
    exact_blocks = math.ceil(exact_budget * 144)
    validated = capabilities.get("spatial_sparse_exact_blocks")
    if not isinstance(validated, (tuple, list)) or exact_blocks not in validated:
        return model, (f"exact_budget={exact_budget:.6g} selects {exact_blocks} blocks, but this build validates "
                       f"sparse blocks {validated}; model returned unchanged")

    clone = model.clone()
    if hasattr(clone, "get_model_object") and hasattr(clone, "add_object_patch"):
        state = PISARuntimeState(armed=True, expected_layers=tuple(range(start_layer, end_layer + 1)))
        clone.set_attachments(PISA_RUNTIME_ATTACHMENT, state)
        try:
            patched = install_anima_pisa_attention(
                clone, native_forward=native.forward_spatial_bhtd, exact_blocks=exact_blocks,
                device_index=device_index, first_layer=start_layer, last_layer=end_layer,
                runtime_state=state if verbose_fallbacks else None)
        except (AttributeError, TypeError, ValueError) as exc:
            return model, f"validated Anima direct PISA integration is unavailable ({exc}); model returned unchanged"
        return clone, (f"model-local B200 direct PISA installed on Anima self-attention blocks {start_layer}:{end_layer} "
                       f"at T=9216; exact_blocks={exact_blocks}; patched_blocks={patched}; "
                       f"runtime_accounting={'enabled' if verbose_fallbacks else 'disabled'}")

    options = clone.model_options.setdefault("transformer_options", {})
    previous = options.get("optimized_attention_override")
    options["optimized_attention_override"] = make_pisa_attention_override(
        exact_budget=exact_budget, allowed_tokens=TOKEN_POLICIES[token_policy], expected_token_shape=ANIMA_TOKEN_SHAPE,
        device_index=device_index, native_forward=native.forward_spatial_bhtd, verbose_fallbacks=verbose_fallbacks,
        previous_override=previous)
    tokens = ",".join(str(x) for x in sorted(TOKEN_POLICIES[token_policy]))
    info = (f"model-local B200 PISA override installed for Anima spatial self-attention at T={tokens}; "
            f"exact_budget={exact_budget:.6g}; layers={start_layer}:{end_layer}")
    if previous is not None:
        info += "; existing optimized_attention_override is chained for fallback"
    return clone, info
