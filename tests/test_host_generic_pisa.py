"""Host logic of the generic PISA override (CPU; the native call is mocked).

Covers the behaviours pinned by the reference's tests/test_generic_pisa.py:
tiling round trips, SD/SDXL/Wan/LTX profiles routed to generic PISA with the
first-order flag and budget clamp, video grids read as 8x8 frame tiles,
dense input stages, every reject reason, backend errors falling back while
out-of-memory stays loud, and the first-call finite check."""
import math
from unittest import mock

import pytest
import torch

from fakes import FakeCudaTensor, OtherDeviceTensor
from rdna35_block_attention.generic_pisa import (MIN_TOKENS, _pack_spatial_blocks, _pack_video_blocks,
                                                 _unpack_spatial_blocks, _unpack_video_blocks,
                                                 make_generic_pisa_override)
from rdna35_block_attention.pisa_runtime import PISARuntimeState

import pisa_oracle as oracle


def _cuda(shape, dtype=torch.float16, cls=FakeCudaTensor):
    return cls(torch.zeros(shape, dtype=dtype))


def _override(previous=None, state=None):
    state = state or PISARuntimeState(armed=True)
    return make_generic_pisa_override(exact_budget=0.25, device_index=0, previous_override=previous,
                                      runtime_state=state), state


def test_spatial_tiling_round_trip_and_matches_kernel_order():
    x = torch.arange(2 * 3 * 256 * 4).reshape(2, 3, 256, 4)
    packed = _pack_spatial_blocks(x, 16)
    assert not torch.equal(packed, x)
    torch.testing.assert_close(_unpack_spatial_blocks(packed, 16), x)
    # the kernels' in-place 8x8 tile order (oracle.ordered_to_raster) is the same permutation
    perm = oracle.raster_permutation(256, 16, 16)
    torch.testing.assert_close(packed, x[:, :, perm])


@pytest.mark.parametrize("grid", [(4, 16, 16), (2, 32, 64)])
def test_video_tiling_round_trip_and_matches_kernel_order(grid):
    t = math.prod(grid)
    x = torch.arange(2 * 3 * t * 4).reshape(2, 3, t, 4)
    packed = _pack_video_blocks(x, grid)
    assert not torch.equal(packed, x)
    torch.testing.assert_close(_unpack_video_blocks(packed, grid), x)
    torch.testing.assert_close(packed, x[:, :, oracle.raster_permutation(t, grid[1], grid[2])])


@pytest.mark.parametrize("profile,heads,head_dim", [("sd15_d40", 8, 40), ("sd15_d80", 8, 80), ("sd15_d160", 8, 160),
                                                    ("sdxl_d64", 10, 64), ("wan_d128", 12, 128), ("ltx_d64", 16, 64)])
def test_flattened_self_attention_profiles_use_generic_pisa(profile, heads, head_dim):
    q = _cuda((1, MIN_TOKENS, heads * head_dim))
    override, state = _override()
    result = torch.zeros((1, heads, MIN_TOKENS, head_dim), dtype=q.dtype)
    with mock.patch("rdna35_block_attention.generic_pisa.generic_pisa_attention",
                    return_value=(result, "b200_0th")) as pisa:
        out = override(mock.Mock(), q, q, q, heads, is_self_attention=True,
                       transformer_options={"block": ("output", 4), "block_index": 1})
    assert out.shape == q.shape
    kwargs = pisa.call_args.kwargs
    first_order = head_dim == 128 and q.dtype == torch.bfloat16
    assert kwargs["use_first_order"] == first_order
    assert kwargs["exact_budget"] == (0.25 if first_order else max(0.25, 0.25))
    assert state.backend_counts["b200_0th"] == 1 and state.per_layer_hits[-1] == 1
    assert state.hit_context_counts["output:4:1"] == 1


@pytest.mark.parametrize("grid", [(2, 64, 64), (4, 32, 64)])
def test_video_grid_passes_frame_tiles_and_keeps_token_order(grid):
    heads, head_dim = 2, 8
    t = math.prod(grid)
    q = FakeCudaTensor(torch.arange(t * heads * head_dim).remainder(1024).to(torch.float16).reshape(1, t, heads * head_dim))
    override, state = _override()

    def identity(q_bhtd, k_bhtd, v_bhtd, **kwargs):
        assert kwargs["token_grid"] == (grid[1], grid[2])
        return q_bhtd, "b200_hyd"

    with mock.patch("rdna35_block_attention.generic_pisa.generic_pisa_attention", side_effect=identity):
        out = override(mock.Mock(), q, q, q, heads, is_self_attention=True, transformer_options={"grid_sizes": grid})
    torch.testing.assert_close(out, q)
    assert state.backend_counts["b200_hyd"] == 1


def test_square_unet_input_stage_stays_dense():
    heads = 10
    q = _cuda((1, 9216, heads * 64))
    previous = mock.Mock(return_value="dense")
    override, state = _override(previous)
    out = override(mock.Mock(), q, q, q, heads, is_self_attention=True,
                   transformer_options={"block": ("input", 4), "block_index": 0})
    assert out == "dense"
    assert state.fallback_reasons["spatial_input_stage_uses_dense_attention"] == 1
    assert sum(state.per_layer_hits.values()) == 0


def test_reject_reasons_chain_previous():
    heads, d = 4, 16
    ok = _cuda((1, MIN_TOKENS, heads * d))
    short = _cuda((1, MIN_TOKENS - 64, heads * d))
    longer = _cuda((1, MIN_TOKENS + 64, heads * d))
    other = _cuda(ok.shape, cls=OtherDeviceTensor)
    bf16 = _cuda(ok.shape, dtype=torch.bfloat16)
    cases = [
        ((ok, ok, ok), {"is_self_attention": False}, "not_explicit_self_attention"),
        ((ok, ok, ok), {"is_self_attention": True, "mask": torch.ones(1)}, "attention_mask_is_not_supported"),
        ((ok, ok, ok), {"is_self_attention": True, "enable_gqa": True}, "gqa_is_not_supported"),
        ((ok, ok, ok), {"is_self_attention": True, "is_kv_cached_attention": True}, "kv_cached_attention_is_not_supported"),
        ((ok, other, other), {"is_self_attention": True}, "qkv_must_share_one_device"),
        ((ok, bf16, bf16), {"is_self_attention": True}, "matching_fp16_or_bf16_qkv_are_required"),
        ((short, short, short), {"is_self_attention": True}, f"tokens_{MIN_TOKENS - 64}_below_{MIN_TOKENS}"),
        ((ok, longer, longer), {"is_self_attention": True}, "matching_btc_qkv_divisible_by_heads_are_required"),
    ]
    previous = mock.Mock(return_value="fallback")
    override, state = _override(previous)
    for tensors, kwargs, reason in cases:
        assert override(mock.Mock(), *tensors, heads, **kwargs) == "fallback"
        assert state.fallback_reasons[reason] == 1, reason
    assert previous.call_count == len(cases)


def test_backend_error_falls_back_but_oom_is_loud():
    heads = 4
    q = _cuda((1, MIN_TOKENS, heads * 16))
    override, state = _override(mock.Mock(return_value="fallback"))
    with mock.patch("rdna35_block_attention.generic_pisa.generic_pisa_attention",
                    side_effect=RuntimeError("launch failed")):
        assert override(mock.Mock(), q, q, q, heads, is_self_attention=True) == "fallback"
    assert state.fallback_reasons["pisa_backend_error_RuntimeError"] == 1
    with mock.patch("rdna35_block_attention.generic_pisa.generic_pisa_attention",
                    side_effect=torch.OutOfMemoryError("out of memory")):
        with pytest.raises(torch.OutOfMemoryError):
            override(mock.Mock(), q, q, q, heads, is_self_attention=True)


def test_nonfinite_first_output_falls_back():
    heads = 4
    q = _cuda((1, MIN_TOKENS, heads * 16))
    override, state = _override(mock.Mock(return_value="fallback"))
    bad = torch.full((1, heads, MIN_TOKENS, 16), torch.nan, dtype=q.dtype)
    with mock.patch("rdna35_block_attention.generic_pisa.generic_pisa_attention", return_value=(bad, "b200_0th")):
        assert override(mock.Mock(), q, q, q, heads, is_self_attention=True) == "fallback"
    assert state.fallback_reasons["pisa_backend_error_ValueError"] == 1
    assert sum(state.per_layer_hits.values()) == 0


@pytest.mark.parametrize("head_dim,dense", [(40, False), (80, False), (64, True)])
def test_small_head_dims_reach_the_native_call_unpadded(head_dim, dense):
    """D < 128 (multiples of 8) reaches the native call as the caller's own
    tensors (no padded copy: the kernels' TMA tiles zero-fill the columns
    past D), with the scale of that D, and the result is returned (into
    ``out`` when given)."""
    from rdna35_block_attention import generic_pisa

    tokens, bh = MIN_TOKENS, 2
    gen = torch.Generator().manual_seed(head_dim)
    q, k, v = (FakeCudaTensor(torch.randn((bh, tokens, head_dim), generator=gen).to(torch.bfloat16)) for _ in range(3))
    seen = {}

    def native_call(qn, kn, vn, *args, **kwargs):
        seen["same"] = qn is q and kn is k and vn is v
        seen["scale"] = args[1] if not dense else args[0]
        result = kwargs.get("out")
        if result is None:
            result = torch.empty((bh, tokens, head_dim), dtype=torch.bfloat16)
        result.copy_(torch.arange(result.numel(), dtype=torch.float32).reshape(result.shape))
        return result

    native = mock.Mock()
    native.generic_forward.side_effect = native_call
    native.full_attention.side_effect = native_call
    out = torch.empty((bh, tokens, head_dim), dtype=torch.bfloat16)
    with mock.patch.object(generic_pisa.device, "native_module", return_value=native):
        got, backend = generic_pisa.generic_pisa_attention(q, k, v, exact_budget=1.0 if dense else 0.125,
                                                           return_backend=True, out=out)
    assert seen["same"]
    assert abs(seen["scale"] - head_dim ** -0.5) < 1e-12
    assert backend == ("dense_b200" if dense else "b200_hyd")
    assert got is out
    expected = torch.arange(bh * tokens * head_dim, dtype=torch.float32).reshape(bh, tokens, head_dim)
    assert torch.equal(out, expected.to(torch.bfloat16))


def test_head_dims_above_128_or_unaligned_are_rejected():
    from rdna35_block_attention import generic_pisa

    for head_dim in (160, 44):
        q = FakeCudaTensor(torch.zeros((1, MIN_TOKENS, head_dim), dtype=torch.bfloat16))
        with pytest.raises(ValueError, match="head_dim"):
            generic_pisa.generic_pisa_attention(q, q, q, exact_budget=0.25)
