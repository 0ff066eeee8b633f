"""Direct per-layer ``attn_op`` patch for the validated Anima model.

Contract kept from the reference's
rdna35_block_attention/anima_pisa_integration.py:21-127 (the names, keyword
signatures, constants and reject-reason strings are the drop-in interface):

* ``validate_anima_pisa_model(patcher)`` raises ValueError unless the
  diffusion model has 28 blocks whose ``self_attn`` is H=16, D=128;
* ``make_anima_pisa_attn_op(original_op, *, native_forward, exact_blocks,
  device_index, layer_index, runtime_state=None)`` returns the replacement
  ``attn_op(q, k, v, transformer_options=None, is_self_attention=False,
  is_initial_transformer_block=None)``: q/k/v are [B,T,H,D]; an eligible
  call (contiguous [B,9216,16,128] BF16 on the validated device, no grad)
  runs ``native_forward`` on BHTD views of the same storage and returns its
  [B,9216,2048] raster output, recording the layer hit; an ineligible call
  records the first failing reason and runs ``original_op``; a native
  failure on an eligible call is recorded and raised as RuntimeError;
* ``install_anima_pisa_attention(patcher, ..., first_layer, last_layer)``
  object-patches layers first..last and returns how many.

Here the eligibility ladder is a table of (check, reason) pairs evaluated in
order, and the replacement op is a small callable object.
"""
from __future__ import annotations

from typing import Any, Callable

import torch

ANIMA_BLOCK_COUNT = 28
ANIMA_PISA_TOKENS = 9216
ANIMA_PISA_HEADS = 16
ANIMA_PISA_HEAD_DIM = 128
ANIMA_PISA_FIRST_LAYER = 20
ANIMA_PISA_LAST_LAYER = 27
_PROFILE = (ANIMA_PISA_TOKENS, ANIMA_PISA_HEADS, ANIMA_PISA_HEAD_DIM)


def validate_anima_pisa_model(model_patcher) -> None:
    blocks = getattr(model_patcher.get_model_object("diffusion_model"), "blocks", None)
    if blocks is None or len(blocks) != ANIMA_BLOCK_COUNT:
        raise ValueError(f"validated Anima model requires {ANIMA_BLOCK_COUNT} blocks")
    for index, block in enumerate(blocks):
        attn = getattr(block, "self_attn", None)
        if attn is None:
            raise ValueError(f"Anima block {index} has no self_attn")
        profile = (getattr(attn, "n_heads", None), getattr(attn, "head_dim", None))
        if profile != (ANIMA_PISA_HEADS, ANIMA_PISA_HEAD_DIM):
            raise ValueError(f"Anima block {index} is not the validated H=16 D=128 attention profile")


def _runtime_shape(q: torch.Tensor) -> tuple[int, int, int, int]:
    """[B,T,H,D] call -> the (B, H, T, D) tuple the runtime report counts."""
    batch, tokens, heads, dim = q.shape
    return batch, heads, tokens, dim


# Eligibility ladder: each entry is (predicate that must hold, reason reported
# when it does not).  Reasons that embed the call's shape are callables.
_LADDER: tuple[tuple[Callable, Any], ...] = (
    (lambda q, k, v, dev: all(isinstance(t, torch.Tensor) for t in (q, k, v)), "qkv_are_not_tensors"),
    (lambda q, k, v, dev: q.ndim == 4 and q.shape == k.shape == v.shape, "matching_bshd_qkv_are_required"),
    (lambda q, k, v, dev: tuple(q.shape[1:]) == _PROFILE,
     lambda q: f"shape_{tuple(q.shape[1:])}_is_not_t9216_h16_d128"),
    (lambda q, k, v, dev: q.dtype == k.dtype == v.dtype == torch.bfloat16, "matching_bfloat16_qkv_are_required"),
    (lambda q, k, v, dev: q.device == k.device == v.device, "qkv_must_share_one_device"),
    (lambda q, k, v, dev: q.device.type == "cuda" and q.device.index == dev, "validated_b200_device_is_required"),
    (lambda q, k, v, dev: all(t.is_contiguous() for t in (q, k, v)), "contiguous_bshd_qkv_are_required"),
    (lambda q, k, v, dev: not any(t.requires_grad for t in (q, k, v)), "forward_only_qkv_are_required"),
)


def _eligible_reason(q, k, v, device_index: int) -> str | None:
    """First failed check of the ladder, or None for an eligible call."""
    for holds, reason in _LADDER:
        if not holds(q, k, v, device_index):
            return reason(q) if callable(reason) else reason
    return None


class _AnimaPisaAttnOp:
    """Replacement attn_op of one Anima block (see the module docstring)."""

    def __init__(self, original_op: Callable, native_forward: Callable, exact_blocks: int, device_index: int,
                 layer_index: int, runtime_state: Any | None):
        self.original_op = original_op
        self.native_forward = native_forward
        self.exact_blocks = exact_blocks
        self.device_index = device_index
        self.layer_index = layer_index
        self.runtime_state = runtime_state

    def _note(self, **event) -> None:
        if self.runtime_state is not None:
            self.runtime_state.record(is_self_attention=True, **event)

    def __call__(self, q, k, v, transformer_options: dict | None = None, is_self_attention: bool = False,
                 is_initial_transformer_block: bool | None = None):
        reason = _eligible_reason(q, k, v, self.device_index)
        if reason is not None:
            self._note(shape=_runtime_shape(q), fallback_reason=reason)
            return self.original_op(q, k, v, transformer_options=transformer_options)
        views = [t.permute(0, 2, 1, 3) for t in (q, k, v)]  # BHTD views of the caller's BTHD storage
        try:
            out = self.native_forward(*views, exact_blocks=self.exact_blocks)
        except Exception as exc:
            self._note(shape=_runtime_shape(q), error=exc)
            raise RuntimeError("RDNA35 PISA (B200) failed for the eligible Anima T=9216 BF16 profile") from exc
        self._note(layer=self.layer_index, shape=_runtime_shape(q))
        return out


def make_anima_pisa_attn_op(original_op: Callable, *, native_forward: Callable, exact_blocks: int, device_index: int,
                            layer_index: int, runtime_state: Any | None = None) -> Callable:
    return _AnimaPisaAttnOp(original_op, native_forward, exact_blocks, device_index, layer_index, runtime_state)


def install_anima_pisa_attention(model_patcher, *, native_forward: Callable, exact_blocks: int, device_index: int,
                                 first_layer: int, last_layer: int, runtime_state: Any | None = None) -> int:
    validate_anima_pisa_model(model_patcher)
    if not 0 <= first_layer <= last_layer < ANIMA_BLOCK_COUNT:
        raise ValueError(f"expected 0 <= first_layer <= last_layer < {ANIMA_BLOCK_COUNT}")
    blocks = model_patcher.get_model_object("diffusion_model").blocks
    patched = range(first_layer, last_layer + 1)
    for index in patched:
        op = make_anima_pisa_attn_op(blocks[index].self_attn.attn_op, native_forward=native_forward,
                                     exact_blocks=exact_blocks, device_index=device_index, layer_index=index,
                                     runtime_state=runtime_state)
        model_patcher.add_object_patch(f"diffusion_model.blocks.{index}.self_attn.attn_op", op)
    return len(patched)
