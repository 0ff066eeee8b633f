"""Pins the CPU oracle (oracle/pisa_oracle.py) -- and the product's CPU-side
helpers -- to golden vectors produced by the reference's own Python code
(tests/golden/make_golden.py)."""
import pathlib

import pytest
import torch

import pisa_oracle as oracle

GOLDEN = torch.load(pathlib.Path(__file__).parent / "golden" / "golden.pt", weights_only=False)


def seeded(shape, seed, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=gen).to(dtype)


@pytest.mark.parametrize("case", GOLDEN["fixed_block"], ids=lambda c: f"causal={c['causal']}")
def test_fixed_block_oracle_matches_reference(case):
    q, k, v = (seeded(case["shape"], s) for s in case["seeds"])
    out = oracle.fixed_block_attention(q, k, v, scale=case["scale"], causal=case["causal"])
    torch.testing.assert_close(out, case["out"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("case", GOLDEN["pisa_hyd"], ids=lambda c: f"T{c['tokens']}_k{c['exact_blocks']}_s{c['sink_block']}")
def test_hyd_oracle_matches_reference_pisa_oracle(case):
    # tolerance of native/rdna35_pisa_ck/tests/test_forward.py:113-117 (the
    # reference's own oracle rounds the centred K to BF16 and merges in one
    # softmax; the restated _forward_impl rounds the exact/tail outputs)
    q, k, v = (seeded((1, case["tokens"], 128), s, torch.bfloat16) for s in case["seeds"])
    out, _ = oracle.hyd_forward(q, k, v, case["exact_blocks"], sink_block=case["sink_block"])
    tol = 6e-2 if case["exact_blocks"] == 0 else 5e-2
    torch.testing.assert_close(out.float(), case["out"].float(), atol=tol, rtol=5e-2)


@pytest.mark.parametrize("case", GOLDEN["pisa_paper"], ids=lambda c: f"T{c['tokens']}")
def test_paper_backend_matches_reference(case):
    from rdna35_block_attention.pisa_attention import pisa_attention

    q, k, v = (seeded((case["bh"], case["tokens"], 128), s, torch.bfloat16) for s in case["seeds"])
    out, info = pisa_attention(q, k, v, exact_blocks=case["exact_blocks"], backend="reference", return_diagnostics=True)
    assert info["backend"] == "reference"
    torch.testing.assert_close(out.float(), case["out"].float(), atol=1.6e-2, rtol=1.6e-2)


def test_tiling_permutations_match_reference_packers():
    from rdna35_block_attention.generic_pisa import _pack_spatial_blocks, _pack_video_blocks

    tiling = GOLDEN["tiling"]
    assert torch.equal(oracle.raster_permutation(256, 16, 16), tiling["spatial_16"])
    assert torch.equal(oracle.raster_permutation(9216, 96, 96), tiling["spatial_96"])
    assert torch.equal(oracle.raster_permutation(2 * 32 * 64, 32, 64), tiling["video_2_32_64"])
    assert torch.equal(_pack_spatial_blocks(torch.arange(256).reshape(1, 1, 256, 1), 16).flatten(), tiling["spatial_16"])
    x = torch.arange(4096).reshape(1, 1, 4096, 1)
    assert torch.equal(_pack_video_blocks(x, (2, 32, 64)).flatten(), tiling["video_2_32_64"])
    # native/rdna35_pisa_ck/tests/test_forward.py:211-224 prefix
    assert oracle.raster_permutation(9216)[:16].tolist() == list(range(8)) + list(range(96, 104))


def test_h3_pack_oracle_matches_reference():
    qkv = torch.arange(1 * 12000 * 3, dtype=torch.float32).reshape(1, 12000, 3, 1, 1)
    views = [qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3)]
    pq, pk, pv, profile = oracle.h3_pack(*views)
    assert profile == GOLDEN["h3_pack"]["profile_12000"]
    assert float(pq.sum() + 2 * pk.sum() + 3 * pv.sum()) == GOLDEN["h3_pack"]["sum"]


def test_hyd_stats_oracle_pins():
    # BF16-max inputs stay finite through the scaled mean (test_forward.py:172-179);
    # v=2000, q=k=0 reproduces v exactly (test_forward.py:164-170)
    q = torch.zeros((1, 128, 128), dtype=torch.bfloat16)
    v = torch.full_like(q, 2000.0)
    out, _ = oracle.hyd_forward(q, q, v, 1)
    assert torch.equal(out, v)
    qc, kc, vc, h_sum, h_norm = oracle.hyd_block_stats(*(seeded((1, 128, 128), 61 + i, torch.bfloat16) for i in range(3)))
    assert qc.dtype == torch.bfloat16 and kc.dtype == torch.float32 and h_norm.shape == (1, 2)


def test_selection_ties_resolve_to_lower_index():
    scores = torch.tensor([[[1.0, 3.0, 3.0, 2.0, 3.0]]])
    assert oracle.select_topk(scores, 2).tolist() == [[[1, 2]]]
    assert oracle.select_topk(scores, 2, sink_block=0).tolist() == [[[0, 1]]]


def block_offset_inputs(tokens, seed, dtype=torch.bfloat16):
    blocks = (tokens + 63) // 64
    base = seeded((1, blocks * 64, 128), seed)
    off = seeded((1, blocks, 1, 128), seed + 100000) * 0.5
    return (base.view(1, blocks, 64, 128) + off).view(1, blocks * 64, 128)[:, :tokens].contiguous().to(dtype)


@pytest.mark.parametrize("case", GOLDEN["pisa_hyd_full"], ids=lambda c: f"T{c['tokens']}_k{c['exact_blocks']}_s{c['sink_block']}")
def test_hyd_oracle_matches_reference_at_full_anima_size(case):
    # 144 blocks with the 23-block cut: the loop oracle and its batched form
    # (the CPU baseline) both agree with the reference's _pisa_reference at
    # its own 5e-2 gate, and with each other exactly
    q, k, v = (block_offset_inputs(case["tokens"], s) for s in case["seeds"])
    stats = oracle.hyd_block_stats(q, k, v)
    batched, idx_b = oracle.hyd_forward_batched(q, k, v, case["exact_blocks"], sink_block=case["sink_block"], stats=stats)
    rows = batched[:, ::case["row_step"]]
    torch.testing.assert_close(rows.float(), case["out_rows"].float(), atol=5e-2, rtol=5e-2)
    loop, idx_l = oracle.hyd_forward(q, k, v, case["exact_blocks"], sink_block=case["sink_block"], stats=stats)
    assert torch.equal(idx_b, idx_l)
    torch.testing.assert_close(batched.float(), loop.float(), atol=1e-2, rtol=1e-2)  # matmul blocking order


@pytest.mark.parametrize("case", GOLDEN["fixed_block_masked"], ids=lambda c: c["name"])
def test_masked_fixed_block_oracle_matches_reference(case):
    """Masked fixed-block attention: the oracle, given the mask broadcast to
    [B,H,T,T] by the reference's rank rules, reproduces the reference's
    outputs, NaN rows included."""
    import make_golden

    q, k, v = (seeded((1, 2, 130, 32), case["seed"] + i) for i in range(3))
    mask = make_golden.make_mask(case)
    if mask.ndim == 3 and mask.shape[0] == 1:  # [B,T,T] with B=1: one mask per batch
        mask = mask[:, None]
    elif mask.ndim == 3:  # [BH,T,T]
        mask = mask.view(1, 2, 130, 130)
    out = oracle.fixed_block_attention(q, k, v, causal=case["causal"], mask=mask)
    assert torch.equal(torch.isnan(out), torch.isnan(case["out"]))
    torch.testing.assert_close(out.nan_to_num(), case["out"].nan_to_num(), atol=1e-5, rtol=1e-5)
