"""GPU end-to-end checks of the drop-in host paths against the CPU oracle:
generic PISA through the ComfyUI override (linear, square-spatial and video
token grids read in place), the MiniMax-H3 native attention on interleaved
views, fixed-block dispatch in every layout, and the pisa_attention router."""
import math
from unittest import mock

import pytest
import torch
import torch.nn.functional as F

import pisa_oracle as oracle
from gpu_util import DEV

pytestmark = pytest.mark.gpu
TOL = dict(atol=5e-2, rtol=5e-2)


def _state():
    from rdna35_block_attention.pisa_runtime import PISARuntimeState

    return PISARuntimeState(armed=True)


@pytest.mark.parametrize("grid", [None, (96, 96), (2, 64, 64)])
def test_generic_override_matches_oracle(grid):
    from rdna35_block_attention.generic_pisa import make_generic_pisa_override

    heads = 2
    # 8320 tokens is not a square, so the linear block order is used
    tokens = 8320 if grid is None else (9216 if len(grid) == 2 else math.prod(grid))
    gen = torch.Generator().manual_seed(tokens + heads)
    q, k, v = (torch.randn((1, tokens, heads * 128), generator=gen).to(torch.bfloat16) for _ in range(3))
    state = _state()
    override = make_generic_pisa_override(exact_budget=0.125, device_index=0, previous_override=None,
                                          runtime_state=state)
    opts = {} if grid is None else ({"grid_sizes": (1, *grid)} if len(grid) == 2 else {"grid_sizes": grid})
    out = override(mock.Mock(), q.to(DEV), k.to(DEV), v.to(DEV), heads, is_self_attention=True,
                   transformer_options=opts).cpu()
    assert state.backend_counts["b200_hyd"] == 1, state.report()
    # oracle: pack into the block order the override uses, run, unpack
    to_bhtd = lambda x: x.view(1, tokens, heads, 128).permute(0, 2, 1, 3)
    if grid is None:
        perm = torch.arange(tokens)
    else:
        perm = oracle.raster_permutation(tokens, grid[-2], grid[-1])
    flat = [to_bhtd(x)[:, :, perm].reshape(heads, tokens, 128).contiguous() for x in (q, k, v)]
    nb = math.ceil(tokens / 64)
    exp, _ = oracle.generic_forward(*flat, math.ceil(0.125 * nb))
    unperm = torch.empty_like(exp)
    unperm[:, perm] = exp
    expected = unperm.view(1, heads, tokens, 128).permute(0, 2, 1, 3).reshape(1, tokens, heads * 128)
    torch.testing.assert_close(out.float(), expected.float(), **TOL)


def test_h3_native_attention_on_interleaved_views():
    from rdna35_block_attention.minimax_h3_gfx1151_attention import minimax_h3_attention

    gen = torch.Generator().manual_seed(4608)
    qkv = torch.randn((1, 700, 3, 4, 128), generator=gen).to(torch.bfloat16)
    views = [qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3)]
    dv = qkv.to(DEV)
    out = minimax_h3_attention(*(dv[:, :, i].permute(0, 2, 1, 3) for i in range(3))).cpu()
    exp, _ = oracle.full_attention(*views)
    torch.testing.assert_close(out.float(), exp.permute(0, 2, 1, 3).reshape(1, 700, 512).float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("layout,dtype", [("bhtd", torch.bfloat16), ("bthd", torch.float16), ("bh_t_d", torch.float32)])
def test_fixed_block_dispatch_layouts(layout, dtype):
    from rdna35_block_attention.dispatch import fixed_block_attention

    gen = torch.Generator().manual_seed(7)
    base = torch.randn((2, 3, 200, 64), generator=gen)
    if layout == "bhtd":
        qkv = [base.to(dtype)] * 3
        kw = {}
    elif layout == "bthd":
        qkv = [base.permute(0, 2, 1, 3).reshape(2, 200, 192).to(dtype)] * 3
        kw = {"heads": 3}
    else:
        qkv = [base.reshape(6, 200, 64).to(dtype)] * 3
        kw = {}
    out, info = fixed_block_attention(*(x.to(DEV) for x in qkv), layout=layout, return_diagnostics=True, **kw)
    assert info["backend"] == "b200", info
    from rdna35_block_attention.reference import fixed_block_attention_ref

    exp = fixed_block_attention_ref(*qkv, layout=layout, **kw)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(out.cpu().float(), exp.float(), atol=tol, rtol=tol)


def test_pisa_attention_router_uses_b200():
    from rdna35_block_attention.pisa_attention import pisa_attention

    q, k, v = oracle.generic_inputs(2, 1024, 3)
    out, info = pisa_attention(q.to(DEV), k.to(DEV), v.to(DEV), exact_blocks=4, return_diagnostics=True)
    assert info["backend"] == "b200" and info["optimized"]
    exp, _ = oracle.hyd_forward(q, k, v, 4)
    torch.testing.assert_close(out.cpu().float(), exp.float(), **TOL)


def test_anima_attn_op_end_to_end():
    from rdna35_block_attention.anima_pisa_integration import make_anima_pisa_attn_op

    import b200_pisa

    q, k, v = oracle.anima_inputs(batch=1, heads=16, seed=5)
    bshd = [x.permute(0, 2, 1, 3).contiguous() for x in (q, k, v)]
    op = make_anima_pisa_attn_op(mock.Mock(), native_forward=b200_pisa.forward_spatial_bhtd, exact_blocks=23,
                                 device_index=0, layer_index=20)
    out = op(*(x.to(DEV) for x in bshd)).cpu()
    exp, _ = oracle.hyd_forward_spatial(q[:, :2], k[:, :2], v[:, :2], 23)
    torch.testing.assert_close(out[:, :, :256].float(), exp.float(), **TOL)


@pytest.mark.parametrize("head_dim,dtype,first_order", [(40, torch.bfloat16, False), (80, torch.bfloat16, False),
                                                        (64, torch.float16, False), (40, torch.bfloat16, True)])
def test_generic_pisa_small_head_dims_match_oracle(head_dim, dtype, first_order):
    # SD1.5-style heads run at their own D (TMA tiles zero-fill the columns past D)
    from rdna35_block_attention.generic_pisa import generic_pisa_attention

    tokens, bh = 8320, 2
    gen = torch.Generator().manual_seed(head_dim)
    q, k, v = (torch.randn((bh, tokens, head_dim), generator=gen).to(dtype) for _ in range(3))
    out, backend = generic_pisa_attention(q.to(DEV), k.to(DEV), v.to(DEV), exact_budget=0.125, return_backend=True,
                                          use_first_order=first_order)
    assert backend == ("b200_hyd" if first_order else "b200_0th")
    assert out.shape == (bh, tokens, head_dim)
    exp, _ = oracle.generic_forward(q, k, v, math.ceil(0.125 * math.ceil(tokens / 64)), use_first_order=first_order)
    torch.testing.assert_close(out.cpu().float(), exp.float(), atol=5e-2, rtol=5e-2)


def test_generic_pisa_small_head_dim_dense_budget_matches_sdpa():
    from rdna35_block_attention.generic_pisa import generic_pisa_attention

    gen = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn((1, 2, 8192, 40), generator=gen).to(torch.bfloat16).to(DEV) for _ in range(3))
    out, backend = generic_pisa_attention(q, k, v, exact_budget=1.0, return_backend=True)
    assert backend == "dense_b200"
    exp = F.scaled_dot_product_attention(q.float(), k.float(), v.float())
    torch.testing.assert_close(out.float(), exp, atol=2e-2, rtol=2e-2)


def test_generic_override_runs_d80_natively_and_d160_falls_back():
    from rdna35_block_attention.generic_pisa import make_generic_pisa_override

    tokens, heads = 8320, 2
    state = _state()
    override = make_generic_pisa_override(exact_budget=0.125, device_index=0, previous_override=None,
                                          runtime_state=state)
    gen = torch.Generator().manual_seed(80)
    q, k, v = (torch.randn((1, tokens, heads * 80), generator=gen).to(torch.bfloat16) for _ in range(3))
    out = override(mock.Mock(), q.to(DEV), k.to(DEV), v.to(DEV), heads, is_self_attention=True).cpu()
    assert state.backend_counts["b200_0th"] == 1, state.report()
    flat = [x.view(1, tokens, heads, 80).permute(0, 2, 1, 3).reshape(heads, tokens, 80) for x in (q, k, v)]
    exact = math.ceil(0.25 * math.ceil(tokens / 64))  # budget clamp max(0.25, .) without first order
    exp, _ = oracle.generic_forward(*flat, exact, use_first_order=False)
    expected = exp.view(1, heads, tokens, 80).permute(0, 2, 1, 3).reshape(1, tokens, heads * 80)
    torch.testing.assert_close(out.float(), expected.float(), atol=5e-2, rtol=5e-2)
    # D=160 exceeds the kernels' 128: the previous backend runs it
    q160 = torch.randn((1, tokens, heads * 160), generator=gen).to(torch.bfloat16).to(DEV)
    original = mock.Mock(return_value="previous")
    assert override(original, q160, q160, q160, heads, is_self_attention=True) == "previous"
    assert any("pisa_backend_error" in r for r in state.fallback_reasons), state.report()


@pytest.mark.parametrize("head_dim", [40, 80, 96])
def test_generic_pisa_small_head_dims_tiled_and_dense(head_dim):
    """D < 128 through the tiled (8x8 per-frame) token order, and dense full
    attention at D = 40 / 80 / 96 on the tcgen05 kernel, against the oracle."""
    import b200_pisa

    gen = torch.Generator().manual_seed(head_dim + 1)
    grid, tokens = (96, 96), 9216
    q, k, v = (torch.randn((1, 2, tokens, head_dim), generator=gen).to(torch.bfloat16) for _ in range(3))
    out = b200_pisa.generic_forward(q.to(DEV), k.to(DEV), v.to(DEV), 23, head_dim ** -0.5, grid=grid).cpu()
    perm = oracle.raster_permutation(tokens, *grid)
    packed = [x[:, :, perm].reshape(2, tokens, head_dim) for x in (q, k, v)]
    exp, _ = oracle.generic_forward(*packed, 23, scale=head_dim ** -0.5)
    unperm = torch.empty_like(exp)
    unperm[:, perm] = exp
    torch.testing.assert_close(out.reshape(2, tokens, head_dim).float(), unperm.float(), atol=5e-2, rtol=5e-2)
    dense = b200_pisa.full_attention(q.to(DEV), k.to(DEV), v.to(DEV), head_dim ** -0.5)
    ref, _ = oracle.full_attention(q, k, v, head_dim ** -0.5)
    torch.testing.assert_close(dense.cpu().float(), ref.float(), atol=2e-2, rtol=2e-2)
