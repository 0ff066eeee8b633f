"""PISA model patch and ``optimized_attention_override`` for B200.

Contract kept from the reference's rdna35_block_attention/pisa_patch.py:41-284
(the public names, keyword signatures, reject-reason strings and the
``(model, info)`` return of the patch function are the drop-in interface):

* ``make_pisa_attention_override(...)`` returns an override
  ``(original_func, q, k, v, heads, mask=None, attn_precision=None,
  skip_reshape=False, skip_output_reshape=False, **kwargs)`` that runs the
  native spatial PISA for explicit, unmasked Anima self-attention on
  pre-reshaped BHTD views of [B,T,H,128] BF16 storage with an enabled token
  count and the (1,96,96) token shape, and otherwise hands the call, with
  all its arguments, to the previous override or the original function;
* ``patch_model_pisa_attention(model, ...)`` validates its arguments and the
  device, then (a) installs the direct per-block ``attn_op`` path when the
  model validates as Anima and the native build supports the requested
  budget, (b) installs this override on a non-ModelPatcher Anima clone, or
  (c) installs the generic PISA override for any other model.  Every refusal
  returns the unchanged model and the reason.

Here the override's eligibility is a table of (check, reason) rows evaluated
in order, and the patch function is split into one helper per outcome.
"""
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
_ANIMA_BLOCKS = 28
_ANIMA_KEY_BLOCKS = 144


def _run_pisa_attention(native_forward: Callable, q, k, v, exact_budget: float, scale: float | None):
    """exact_blocks = ceil(budget * blocks), capped at the block count."""
    blocks = -(-q.shape[-2] // 64)
    return native_forward(q, k, v, min(blocks, math.ceil(exact_budget * blocks)), scale=scale)


def _fallback_call(previous_override: Callable | None, original_func: Callable, *args, **kwargs):
    if previous_override is None:
        return original_func(*args, **kwargs)
    return previous_override(original_func, *args, **kwargs)


def _device_index() -> tuple[int | None, str | None]:
    return device.b200_device_index()


def _square_side_ok(tokens: int) -> bool:
    side = math.isqrt(tokens)
    return side * side == tokens and side % SPATIAL_BLOCK_EDGE == 0


def _raster_strides_ok(q, k, v) -> bool:
    _, heads, tokens, dim = q.shape
    want = (heads * tokens * dim, dim, heads * dim, 1)
    return all(t.stride() == want for t in (q, k, v))


# (check, reason) rows; a check sees one namespace `c` of the call.  Reasons
# that quote the call are callables of `c`.
_LADDER: tuple[tuple[Callable, Any], ...] = (
    (lambda c: c.kwargs.get("is_self_attention") is True, "call_is_not_explicitly_self_attention"),
    (lambda c: c.mask is None, "attention_mask_is_not_supported"),
    (lambda c: bool(c.skip_reshape), "pre_reshaped_qkv_is_required"),
    (lambda c: not c.skip_output_reshape, "merged_attention_output_is_required"),
    (lambda c: all(isinstance(t, torch.Tensor) for t in c.qkv), "qkv_are_not_tensors"),
    (lambda c: c.q.ndim == 4 and c.q.shape == c.k.shape == c.v.shape, "matching_bhtd_qkv_are_required"),
    (lambda c: c.q.shape[0] > 0 and c.q.shape[1] == c.heads and c.q.shape[-1] == 128,
     "unsupported_batch_heads_or_head_dim"),
    (lambda c: c.q.shape[-2] in c.allowed_tokens, lambda c: f"tokens_{c.q.shape[-2]}_are_not_enabled"),
    (lambda c: isinstance(c.token_shape, (tuple, list)) and tuple(c.token_shape) == c.expected_token_shape,
     lambda c: f"token_shape_{c.token_shape}_is_not_{c.expected_token_shape}"),
    (lambda c: _square_side_ok(c.q.shape[-2]), "square_spatial_tokens_divisible_by_8_are_required"),
    (lambda c: c.kwargs.get("is_initial_transformer_block") is False, "initial_or_unmarked_transformer_block"),
    (lambda c: c.q.dtype == c.k.dtype == c.v.dtype == torch.bfloat16, "matching_bfloat16_qkv_are_required"),
    (lambda c: c.q.device == c.k.device == c.v.device, "qkv_must_share_one_device"),
    (lambda c: c.q.device.type == "cuda", "cuda_device_is_required"),
    (lambda c: c.q.device.index == c.device_index,
     lambda c: f"cuda_device_{c.q.device.index}_is_not_validated_device_{c.device_index}"),
    (lambda c: _raster_strides_ok(c.q, c.k, c.v), "bhtd_views_over_contiguous_bthd_storage_are_required"),
    (lambda c: not any(t.requires_grad for t in c.qkv), "forward_only_qkv_are_required"),
    (lambda c: c.attn_precision != torch.float32, "float32_attention_precision_is_not_supported"),
    (lambda c: not c.kwargs.get("enable_gqa", False), "gqa_is_not_supported"),
)


class _Call:
    """The arguments of one override call, as the ladder reads them."""

    def __init__(self, q, k, v, heads, mask, attn_precision, skip_reshape, skip_output_reshape, allowed_tokens,
                 expected_token_shape, device_index, kwargs):
        self.q, self.k, self.v, self.qkv = q, k, v, (q, k, v)
        self.heads, self.mask, self.attn_precision = heads, mask, attn_precision
        self.skip_reshape, self.skip_output_reshape = skip_reshape, skip_output_reshape
        self.allowed_tokens, self.expected_token_shape = allowed_tokens, expected_token_shape
        self.device_index, self.kwargs = device_index, kwargs
        self.token_shape = kwargs.get("attention_token_shape")


def _pisa_reject_reason(q, k, v, heads, mask, attn_precision, skip_reshape, skip_output_reshape,
                        allowed_tokens: frozenset, expected_token_shape: tuple, device_index: int,
                        kwargs: dict[str, Any]) -> str | None:
    call = _Call(q, k, v, heads, mask, attn_precision, skip_reshape, skip_output_reshape, allowed_tokens,
                 expected_token_shape, device_index, kwargs)
    for holds, reason in _LADDER:
        if not holds(call):
            return reason(call) if callable(reason) else reason
    return None


def make_pisa_attention_override(*, exact_budget: float, allowed_tokens: frozenset, expected_token_shape: tuple,
                                 device_index: int, native_forward: Callable, verbose_fallbacks: bool,
                                 previous_override: Callable | None) -> Callable:
    def attention_override(original_func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                           skip_output_reshape=False, **kwargs):
        reason = _pisa_reject_reason(q, k, v, heads, mask, attn_precision, skip_reshape, skip_output_reshape,
                                     allowed_tokens, expected_token_shape, device_index, kwargs)
        if reason is None:
            return _run_pisa_attention(native_forward, q, k, v, exact_budget, kwargs.get("scale"))
        if verbose_fallbacks:
            logging.info("%s: original attention used: %s", LOG_PREFIX, reason)
        return _fallback_call(previous_override, original_func, q, k, v, heads, mask=mask,
                              attn_precision=attn_precision, skip_reshape=skip_reshape,
                              skip_output_reshape=skip_output_reshape, **kwargs)

    return attention_override


def _arguments_problem(model, exact_budget, token_policy, start_layer, end_layer) -> str | None:
    if not 0.0 <= exact_budget <= 1.0:
        return f"invalid exact_budget={exact_budget}"
    if token_policy not in TOKEN_POLICIES:
        return f"unsupported token_policy={token_policy}"
    if not 0 <= start_layer <= end_layer < _ANIMA_BLOCKS:
        return f"invalid Anima layer range {start_layer}:{end_layer}"
    if not (hasattr(model, "clone") and hasattr(model, "model_options")):
        return "MODEL does not expose ComfyUI ModelPatcher clone/model_options"
    return None


def _validates_as_anima(model) -> bool:
    if not (hasattr(model, "get_model_object") and hasattr(model, "add_object_patch")):
        return False
    try:
        validate_anima_pisa_model(model)
    except (AttributeError, TypeError, ValueError):
        return False
    return True


def _chained_note(previous) -> str:
    return "; existing optimized_attention_override is chained for fallback" if previous is not None else ""


def _install_generic(model, exact_budget, device_index, verbose_fallbacks):
    clone = model.clone()
    state = PISARuntimeState(armed=True)
    if hasattr(clone, "set_attachments"):
        clone.set_attachments(PISA_RUNTIME_ATTACHMENT, state)
    options = clone.model_options.setdefault("transformer_options", {})
    previous = options.get("optimized_attention_override")
    options["optimized_attention_override"] = make_generic_pisa_override(
        exact_budget=exact_budget, device_index=device_index, previous_override=previous, runtime_state=state,
        validate_output=verbose_fallbacks)
    return clone, ("model-local generic B200 PISA installed for explicit self-attention with T>=8192"
                   + _chained_note(previous))


def _load_native(exact_budget):
    """(native module, exact_blocks, None) or (None, None, refusal reason)."""
    try:
        native = importlib.import_module("b200_pisa")
        build_info, capabilities = native.build_info(), native.capabilities()
        native.prepare()
    except (ImportError, OSError, RuntimeError, AttributeError) as exc:
        return None, None, f"b200_pisa is unavailable ({type(exc).__name__}: {exc})"
    if build_info.get("api") != NATIVE_API:
        return None, None, f"b200_pisa API {NATIVE_API} is required, got {build_info.get('api')}"
    exact_blocks = math.ceil(exact_budget * _ANIMA_KEY_BLOCKS)
    validated = capabilities.get("spatial_sparse_exact_blocks")
    if not isinstance(validated, (tuple, list)) or exact_blocks not in validated:
        return None, None, (f"exact_budget={exact_budget:.6g} selects {exact_blocks} blocks, but this build "
                            f"validates sparse blocks {validated}")
    return native, exact_blocks, None


def _install_direct(model, clone, native, exact_blocks, device_index, start_layer, end_layer, verbose_fallbacks):
    state = PISARuntimeState(armed=True, expected_layers=tuple(range(start_layer, end_layer + 1)))
    clone.set_attachments(PISA_RUNTIME_ATTACHMENT, state)
    try:
        patched = install_anima_pisa_attention(
            clone, native_forward=native.forward_spatial_bhtd, exact_blocks=exact_blocks, device_index=device_index,
            first_layer=start_layer, last_layer=end_layer, runtime_state=state if verbose_fallbacks else None)
    except (AttributeError, TypeError, ValueError) as exc:
        return model, f"validated Anima direct PISA integration is unavailable ({exc}); model returned unchanged"
    accounting = "enabled" if verbose_fallbacks else "disabled"
    return clone, (f"model-local B200 direct PISA installed on Anima self-attention blocks {start_layer}:{end_layer} "
                   f"at T=9216; exact_blocks={exact_blocks}; patched_blocks={patched}; "
                   f"runtime_accounting={accounting}")


def _install_override(clone, native, exact_budget, token_policy, device_index, start_layer, end_layer,
                      verbose_fallbacks):
    options = clone.model_options.setdefault("transformer_options", {})
    previous = options.get("optimized_attention_override")
    options["optimized_attention_override"] = make_pisa_attention_override(
        exact_budget=exact_budget, allowed_tokens=TOKEN_POLICIES[token_policy], expected_token_shape=ANIMA_TOKEN_SHAPE,
        device_index=device_index, native_forward=native.forward_spatial_bhtd, verbose_fallbacks=verbose_fallbacks,
        previous_override=previous)
    tokens = ",".join(map(str, sorted(TOKEN_POLICIES[token_policy])))
    return clone, (f"model-local B200 PISA override installed for Anima spatial self-attention at T={tokens}; "
                   f"exact_budget={exact_budget:.6g}; layers={start_layer}:{end_layer}" + _chained_note(previous))


def patch_model_pisa_attention(model, *, enabled: bool, exact_budget: float, token_policy: str,
                               verbose_fallbacks: bool, start_layer: int = ANIMA_PISA_FIRST_LAYER,
                               end_layer: int = ANIMA_PISA_LAST_LAYER):
    unchanged = "; model returned unchanged"
    if not enabled:
        return model, "disabled" + unchanged
    problem = _arguments_problem(model, exact_budget, token_policy, start_layer, end_layer)
    if problem is not None:
        return model, problem + unchanged
    device_index, device_error = _device_index()
    if device_index is None:
        return model, f"{device_error}" + unchanged
    if not _validates_as_anima(model):
        return _install_generic(model, exact_budget, device_index, verbose_fallbacks)
    native, exact_blocks, refusal = _load_native(exact_budget)
    if refusal is not None:
        return model, refusal + unchanged
    clone = model.clone()
    if hasattr(clone, "get_model_object") and hasattr(clone, "add_object_patch"):
        return _install_direct(model, clone, native, exact_blocks, device_index, start_layer, end_layer,
                               verbose_fallbacks)
    return _install_override(clone, native, exact_budget, token_policy, device_index, start_layer, end_layer,
                             verbose_fallbacks)
