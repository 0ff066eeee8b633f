"""Generic PISA for image/video self-attention with T >= 8192 (mirrors the
reference's rdna35_block_attention/generic_pisa.py:17-391 contract: the same
override signature, reject reasons, spatial/video token tiling rules,
first-call finite check, fallback on backend errors except out-of-memory).

On B200 the whole path is one native call (``b200_pisa.generic_forward``):
statistics, routing, exact block-sparse attention, centroid tail and
first-order correction, reading 8x8 spatial/video tiles in place through
strided views instead of packing copies."""
from __future__ import annotations

import math
from typing import Callable

import torch
import torch.nn.functional as F

from . import device

BLOCK_SIZE = 64
MIN_TOKENS = 8192
NATIVE_HEAD_DIM = 128  # the kernels' tile width; smaller heads are zero-filled by the TMA loads
SPATIAL_BLOCK_EDGE = 8


# ---- token tiling helpers (the reference's generic_pisa.py:17-52 names).
# Block-major order of a frame of H x W tokens: 8x8 tiles in raster order of
# the tiles, each tile's 64 tokens in raster order inside the tile.  Here the
# order is an index map, applied with one gather (pack) or scatter (unpack)
# along the token axis; the kernels read the same order in place through
# strided views, so these copies serve callers that want block-major tensors.
def _block_order(height: int, width: int, device=None) -> torch.Tensor:
    """raster index of the token at each block-major position of one frame."""
    if height % SPATIAL_BLOCK_EDGE or width % SPATIAL_BLOCK_EDGE:
        raise ValueError("spatial grid sides must be multiples of 8")
    e = SPATIAL_BLOCK_EDGE
    pos = torch.arange(height * width, device=device)
    tile, inner = pos // (e * e), pos % (e * e)
    tiles_per_row = width // e
    row = (tile // tiles_per_row) * e + inner // e
    col = (tile % tiles_per_row) * e + inner % e
    return row * width + col


def _frames_order(frames: int, height: int, width: int, device=None) -> torch.Tensor:
    frame = height * width
    base = _block_order(height, width, device)
    return (torch.arange(frames, device=device)[:, None] * frame + base[None]).reshape(-1)


def _gather_tokens(tensor, order: torch.Tensor):
    return tensor.index_select(-2, order.to(tensor.device)).contiguous()


def _scatter_tokens(tensor, order: torch.Tensor):
    out = torch.empty_like(tensor)
    out[..., order.to(tensor.device), :] = tensor
    return out


def _pack_spatial_blocks_2d(tensor, height: int, width: int):
    return _gather_tokens(tensor, _block_order(height, width))


def _unpack_spatial_blocks_2d(tensor, height: int, width: int):
    return _scatter_tokens(tensor, _block_order(height, width))


def _pack_spatial_blocks(tensor, side: int):
    return _pack_spatial_blocks_2d(tensor, side, side)


def _unpack_spatial_blocks(tensor, side: int):
    return _unpack_spatial_blocks_2d(tensor, side, side)


def _check_video(tensor, grid_sizes):
    frames, height, width = grid_sizes
    if tensor.shape[-2] != frames * height * width:
        raise ValueError("video token shape does not match grid_sizes")


def _pack_video_blocks(tensor, grid_sizes):
    _check_video(tensor, grid_sizes)
    return _gather_tokens(tensor, _frames_order(*grid_sizes))


def _unpack_video_blocks(tensor, grid_sizes):
    _check_video(tensor, grid_sizes)
    return _scatter_tokens(tensor, _frames_order(*grid_sizes))


def generic_pisa_attention(q, k, v, *, exact_budget: float, scale: float | None = None, return_backend: bool = False,
                           use_first_order: bool = True, debug_finite: bool = False,
                           token_grid: tuple[int, int] | None = None, out=None):
    """PISA over [BH,T,D] (or [B,H,T,D]) fp16/bf16 q/k/v on one CUDA device,
    D <= 128 in multiples of 8 (the reference's generic path accepts any D;
    D > 128, e.g. SD1.5's 160, stays with the previous backend).
    token_grid=(h, w): tokens are per-frame h x w rasters read in 8x8-tile
    block order; the output stays in token order."""
    if q.ndim not in (3, 4) or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("generic PISA requires matching [BH,T,D] q/k/v")
    tokens, head_dim = q.shape[-2], q.shape[-1]
    if tokens < MIN_TOKENS:
        raise ValueError(f"generic PISA requires at least {MIN_TOKENS} tokens")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("generic PISA requires matching fp16/bf16 q/k/v")
    if not q.is_cuda or q.device != k.device or q.device != v.device:
        raise ValueError("generic PISA requires q/k/v on one CUDA device")
    if head_dim > NATIVE_HEAD_DIM or head_dim % 8:
        raise ValueError(f"B200 generic PISA supports head_dim <= {NATIVE_HEAD_DIM} in multiples of 8")
    blocks = math.ceil(tokens / BLOCK_SIZE)
    exact_blocks = min(blocks, max(1, math.ceil(exact_budget * blocks)))
    scale_value = float(scale) if scale is not None else 1.0 / math.sqrt(head_dim)
    native = device.native_module()
    # SD1.5 / SDXL heads (D = 40, 64, 80 ...) run at their own D: the
    # kernels' 128-wide TMA tiles load the columns past D as zeros, which
    # changes no dot product, centroid, routing score or first-order term
    if exact_blocks == blocks:
        output = native.full_attention(q, k, v, scale_value, out=out)
        return (output, "dense_b200") if return_backend else output
    output = native.generic_forward(q, k, v, exact_blocks, scale_value, first_order=use_first_order,
                                    grid=token_grid, out=out)
    if debug_finite and not torch.isfinite(output).all().item():
        raise ValueError("generic PISA non-finite stages: output")
    backend = "b200_hyd" if use_first_order else "b200_0th"
    return (output, backend) if return_backend else output


# Call-level reject ladder of the generic override: (check, reason) rows in
# order, the first failing row names the reason (reason strings kept from
# the reference's generic override).
_CALL_LADDER = (
    (lambda q, k, v, mask, dev, kw: kw.get("is_self_attention") is True, "not_explicit_self_attention"),
    (lambda q, k, v, mask, dev, kw: not kw.get("is_kv_cached_attention", False), "kv_cached_attention_is_not_supported"),
    (lambda q, k, v, mask, dev, kw: mask is None, "attention_mask_is_not_supported"),
    (lambda q, k, v, mask, dev, kw: not kw.get("enable_gqa", False), "gqa_is_not_supported"),
    (lambda q, k, v, mask, dev, kw: all(isinstance(t, torch.Tensor) for t in (q, k, v)), "qkv_are_not_tensors"),
    (lambda q, k, v, mask, dev, kw: q.device.type == "cuda" and q.device.index == dev,
     "validated_b200_device_is_required"),
    (lambda q, k, v, mask, dev, kw: k.device == q.device == v.device, "qkv_must_share_one_device"),
    (lambda q, k, v, mask, dev, kw: q.dtype in (torch.float16, torch.bfloat16) and k.dtype == q.dtype == v.dtype,
     "matching_fp16_or_bf16_qkv_are_required"),
)


def _call_reject_reason(q, k, v, mask, device_index, kwargs) -> str | None:
    for holds, reason in _CALL_LADDER:
        if not holds(q, k, v, mask, device_index, kwargs):
            return reason
    return None


def _bhtd_layout(q, k, v, heads, skip_reshape):
    """((q, k, v) as [B,H,T,D] views, (B, T, D)) of ComfyUI's two input
    layouts, or the reject reason when the tensors do not fit the layout."""
    if skip_reshape:  # [B,H,T,D]
        if q.ndim != 4 or not (q.shape == k.shape == v.shape):
            return "matching_bhtd_qkv_are_required"
        if q.shape[1] != heads:
            return "head_count_mismatch"
        return (q, k, v), (q.shape[0], q.shape[2], q.shape[3])
    if q.ndim != 3 or not (q.shape == k.shape == v.shape) or q.shape[-1] % heads:  # [B,T,H*D]
        return "matching_btc_qkv_divisible_by_heads_are_required"
    batch, tokens, channels = q.shape
    head_dim = channels // heads
    return tuple(t.unflatten(2, (heads, head_dim)).transpose(1, 2) for t in (q, k, v)), (batch, tokens, head_dim)


def make_generic_pisa_override(*, exact_budget: float, device_index: int, previous_override: Callable | None,
                               runtime_state, validate_output: bool = False) -> Callable:
    def fallback(original_func, *args, **kwargs):
        if previous_override is not None:
            return previous_override(original_func, *args, **kwargs)
        return original_func(*args, **kwargs)

    def attention_override(original_func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                           skip_output_reshape=False, **kwargs):
        call = dict(mask=mask, attn_precision=attn_precision, skip_reshape=skip_reshape,
                    skip_output_reshape=skip_output_reshape, **kwargs)
        options = kwargs.get("transformer_options") or {}
        block = options.get("block")
        block_index = options.get("block_index", 0)
        context = f"{block[0]}:{block[1]}:{block_index}" if isinstance(block, (tuple, list)) and len(block) == 2 else None
        reason = _call_reject_reason(q, k, v, mask, device_index, kwargs)
        if reason is None:
            layout = _bhtd_layout(q, k, v, heads, skip_reshape)
            if isinstance(layout, str):
                reason = layout
            else:
                (q_bhtd, k_bhtd, v_bhtd), (batch, tokens, head_dim) = layout
                if tokens < MIN_TOKENS:
                    reason = f"tokens_{tokens}_below_{MIN_TOKENS}"
        shape = tuple(q.shape) if isinstance(q, torch.Tensor) and q.ndim >= 2 else None
        if reason is not None:
            runtime_state.record(is_self_attention=kwargs.get("is_self_attention"), shape=shape,
                                 fallback_reason=reason, context=context)
            return fallback(original_func, q, k, v, heads, **call)

        grid_sizes = options.get("attention_token_grid", options.get("grid_sizes"))
        video = (isinstance(grid_sizes, (tuple, list)) and len(grid_sizes) == 3
                 and all(isinstance(x, int) and x > 0 for x in grid_sizes) and math.prod(grid_sizes) == tokens
                 and grid_sizes[1] % SPATIAL_BLOCK_EDGE == 0 and grid_sizes[2] % SPATIAL_BLOCK_EDGE == 0)
        side = math.isqrt(tokens)
        spatial = side * side == tokens and side % SPATIAL_BLOCK_EDGE == 0
        if spatial and isinstance(block, (tuple, list)) and block[0] == "input":
            reason = "spatial_input_stage_uses_dense_attention"
            runtime_state.record(is_self_attention=True, shape=(batch, heads, tokens, head_dim),
                                 fallback_reason=reason, context=context)
            return fallback(original_func, q, k, v, heads, **call)
        token_grid = (grid_sizes[1], grid_sizes[2]) if video else ((side, side) if spatial else None)
        use_first_order = head_dim == 128 and q.dtype == torch.bfloat16
        budget = exact_budget if use_first_order else max(0.25, exact_budget)
        if skip_output_reshape:
            out = q.new_empty((batch, heads, tokens, head_dim))
            out_view = out
        else:
            out = q.new_empty((batch, tokens, heads * head_dim))
            out_view = out.view(batch, tokens, heads, head_dim).transpose(1, 2)
        try:
            output, backend = generic_pisa_attention(q_bhtd, k_bhtd, v_bhtd, exact_budget=budget,
                                                     scale=kwargs.get("scale"), return_backend=True,
                                                     use_first_order=use_first_order, debug_finite=validate_output,
                                                     token_grid=token_grid, out=out_view)
            profile = (backend, batch, heads, tokens, head_dim, str(q.dtype))
            if not runtime_state.is_profile_validated(profile):
                if not torch.isfinite(output).all().item():
                    raise ValueError("generic PISA produced non-finite output")
                runtime_state.mark_profile_validated(profile)
        except (RuntimeError, ValueError, NotImplementedError) as exc:
            if isinstance(exc, torch.OutOfMemoryError):
                raise
            reason = f"pisa_backend_error_{type(exc).__name__}"
            runtime_state.record(is_self_attention=True, shape=(batch, heads, tokens, head_dim),
                                 fallback_reason=reason, context=context, error=exc if validate_output else None)
            return fallback(original_func, q, k, v, heads, **call)
        quality = None
        if validate_output and runtime_state.quality_sample is None:
            ref = F.scaled_dot_product_attention(q_bhtd, k_bhtd, v_bhtd, scale=kwargs.get("scale")).float()
            got = output.float() if output.shape == ref.shape else out_view.float()
            cosine = F.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
            mae = (got - ref).abs().mean().item()
            quality = (f"cos={cosine:.6f},mae={mae:.6g},pisa_max={got.abs().max().item():.6g},"
                       f"sdpa_max={ref.abs().max().item():.6g}")
        runtime_state.record(layer=-1, is_self_attention=True, shape=(batch, heads, tokens, head_dim),
                             backend=backend, context=context, quality=quality)
        if output is out_view or output.data_ptr() == out.data_ptr():
            return out
        # a replacement backend returned its own tensor ([B,H,T,D] in token order)
        output = output.reshape(batch, heads, tokens, head_dim)
        return output if skip_output_reshape else output.transpose(1, 2).contiguous().flatten(2)

    return attention_override
