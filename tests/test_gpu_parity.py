"""GPU parity of every C-ABI kernel family against the CPU oracle."""
import math

import pytest
import torch
import torch.nn.functional as F

import pisa_oracle as oracle
from gpu_util import DEV, to_dev_bhtd

pytestmark = pytest.mark.gpu

TOL = dict(atol=5e-2, rtol=5e-2)  # BF16 gate of native/rdna35_pisa_ck/tests/test_forward.py:113-117


@pytest.fixture(scope="module")
def pisa():
    import b200_pisa

    b200_pisa.prepare()
    return b200_pisa


def _bh_inputs(bh, tokens, seed, dtype=torch.bfloat16):
    q, k, v = oracle.generic_inputs(bh, tokens, seed, dtype)
    return (q, k, v), tuple(x.to(DEV) for x in (q, k, v))


@pytest.mark.parametrize("tokens", [64, 65, 128, 1000, 9216])
def test_hyd_stats_match_oracle(pisa, tokens):
    (q, k, v), (qd, kd, vd) = _bh_inputs(2, tokens, 11)
    got = pisa._C.block_stats_hyd(qd, kd, vd)
    exp = oracle.hyd_block_stats(q, k, v)
    # centroids: same sequential FP32 sums and 1/len multiply -> bit-exact
    for i in range(3):
        torch.testing.assert_close(got[i].cpu(), exp[i], atol=0, rtol=0)
    torch.testing.assert_close(got[3].cpu(), exp[3], atol=2e-3, rtol=1e-4)
    torch.testing.assert_close(got[4].cpu(), exp[4], atol=1e-2, rtol=1e-3)


def test_hyd_stats_centring_large_offsets(pisa):
    # test_forward.py:127-137 pattern: K = offset 64 + noise 0.125
    torch.manual_seed(37)
    tokens = 256
    offsets = torch.randn((1, tokens // 64, 1, 128)) * 64.0
    noise = torch.randn((1, tokens // 64, 64, 128)) * 0.125
    k = (offsets + noise).flatten(1, 2).to(torch.bfloat16)
    q = (torch.randn((1, tokens, 128)) * 16).to(torch.bfloat16)
    v = torch.randn_like(k)
    got = pisa._C.block_stats_hyd(q.to(DEV), k.to(DEV), v.to(DEV))
    exp = oracle.hyd_block_stats(q, k, v)
    torch.testing.assert_close(got[3].cpu(), exp[3], atol=1e-3, rtol=1e-4)
    torch.testing.assert_close(got[4].cpu(), exp[4], atol=1e-3, rtol=1e-4)


def test_block_stats_extrema_finite(pisa):
    # test_forward.py:172-179: BF16-max inputs average without overflow
    maximum = torch.finfo(torch.bfloat16).max
    q = torch.full((1, 65, 128), maximum, device=DEV, dtype=torch.bfloat16)
    for t in pisa._C.block_stats(q, q, q):
        assert torch.isfinite(t).all() and (t > 0).all()


@pytest.mark.parametrize("tokens,exact", [(128, 1), (65, 1), (256, 2), (9216, 23), (4096, 10)])
def test_hyd_forward_matches_oracle(pisa, tokens, exact):
    (q, k, v), (qd, kd, vd) = _bh_inputs(2, tokens, 19)
    got = pisa.forward(qd, kd, vd, exact_blocks=exact).cpu().float()
    exp, _ = oracle.hyd_forward(q, k, v, exact)
    torch.testing.assert_close(got, exp.float(), **TOL)


@pytest.mark.parametrize("sink", [0, -1])
def test_hyd_forward_sink(pisa, sink):
    (q, k, v), (qd, kd, vd) = _bh_inputs(1, 65, 23)
    got = pisa.forward(qd, kd, vd, exact_blocks=1, sink_block=sink).cpu().float()
    exp, _ = oracle.hyd_forward(q, k, v, 1, sink_block=sink)
    torch.testing.assert_close(got, exp.float(), **TOL)


def test_hyd_forward_zero_exact_blocks(pisa):
    torch.manual_seed(37)
    tokens = 256
    q = (torch.randn((1, tokens, 128)) * 16.0).to(torch.bfloat16)
    offsets = torch.randn((1, tokens // 64, 1, 128)) * 64.0
    noise = torch.randn((1, tokens // 64, 64, 128)) * 0.125
    k = (offsets + noise).flatten(1, 2).to(torch.bfloat16)
    v = torch.randn_like(k)
    got = pisa.forward(q.to(DEV), k.to(DEV), v.to(DEV), exact_blocks=0).cpu().float()
    exp, _ = oracle.hyd_forward(q, k, v, 0)
    torch.testing.assert_close(got, exp.float(), atol=6e-2, rtol=5e-2)


def test_dense_exact_matches_sdpa(pisa):
    (q, k, v), (qd, kd, vd) = _bh_inputs(1, 128, 17)
    got = pisa.forward(qd, kd, vd, exact_blocks=2, scale=0.125)
    exp = F.scaled_dot_product_attention(qd[:, None], kd[:, None], vd[:, None], scale=0.125).squeeze(1)
    torch.testing.assert_close(got, exp, atol=2e-2, rtol=2e-2)


def test_large_values_stay_finite(pisa):
    q = torch.zeros((1, 128, 128), device=DEV, dtype=torch.bfloat16)
    v = torch.full_like(q, 2000.0)
    out = pisa.forward(q, torch.zeros_like(q), v, exact_blocks=1)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out, v, atol=0.0, rtol=0.0)


def test_spatial_forward_matches_oracle(pisa):
    from b200_pisa import _lib

    q, k, v = oracle.anima_inputs(batch=1, heads=2, seed=3)
    got = pisa.forward_spatial_bhtd(*(to_dev_bhtd(x) for x in (q, k, v)), exact_blocks=23)
    assert _lib.last_kernel() == "tcgen05"
    assert _lib.read_status() == 0
    got = got.cpu().float()
    exp, _ = oracle.hyd_forward_spatial(q, k, v, 23)
    assert got.shape == (1, 9216, 256)
    torch.testing.assert_close(got, exp.float(), **TOL)


def test_spatial_dense_matches_sdpa(pisa):
    q, k, v = oracle.anima_inputs(batch=1, heads=2, seed=43)
    qd, kd, vd = (to_dev_bhtd(x) for x in (q, k, v))
    got = pisa.forward_spatial_bhtd(qd, kd, vd, exact_blocks=144)
    exp = F.scaled_dot_product_attention(qd, kd, vd).permute(0, 2, 1, 3).reshape(1, 9216, 256)
    torch.testing.assert_close(got, exp, atol=2e-2, rtol=2e-2)


def test_spatial_pack_unpack_round_trip(pisa):
    batch, heads, tokens = 1, 2, 9216
    raster = torch.arange(tokens, device=DEV, dtype=torch.float32).to(torch.bfloat16)
    base = raster.view(1, tokens, 1, 1).expand(batch, tokens, heads, 128).contiguous()
    bhtd = base.permute(0, 2, 1, 3)
    pq, pk, pv = pisa._C.pack_spatial_qkv(bhtd, bhtd, bhtd)
    assert pq[0, :16, 0].float().tolist() == list(range(8)) + list(range(96, 104))
    torch.testing.assert_close(pq, pk, atol=0, rtol=0)
    restored = pisa._C.unpack_spatial_output(pq, batch, heads)
    torch.testing.assert_close(restored, base.flatten(2), atol=0, rtol=0)


def test_spatial_epilogue_matches_merge(pisa):
    batch, heads, tokens = 1, 2, 9216
    torch.manual_seed(53)
    exact = torch.randn((2, tokens, 128), dtype=torch.bfloat16)
    approx = torch.randn_like(exact)
    corr = torch.randn((2, tokens, 128))
    le = torch.randn((2, tokens))
    la = torch.randn((2, tokens))
    got = pisa._C.fuse_spatial_epilogue(exact.to(DEV), le.to(DEV), approx.to(DEV), la.to(DEV), corr.to(DEV), batch, heads)
    exp = oracle.unpack_spatial(oracle.merge_epilogue(exact, le, approx, la, corr), batch, heads)
    torch.testing.assert_close(got.cpu(), exp, atol=0.03125, rtol=0.0)


@pytest.mark.parametrize("tq,tk,d", [(1000, 1000, 128), (9216, 512, 128), (333, 777, 64)])
def test_full_attention_matches_oracle(pisa, tq, tk, d):
    gen = torch.Generator().manual_seed(tq + tk)
    q = torch.randn((2, 3, tq, d), generator=gen).to(torch.bfloat16)
    k = torch.randn((2, 3, tk, d), generator=gen).to(torch.bfloat16)
    v = torch.randn((2, 3, tk, d), generator=gen).to(torch.bfloat16)
    got = pisa.full_attention(q.to(DEV), k.to(DEV), v.to(DEV), 1 / math.sqrt(d)).cpu().float()
    exp, _ = oracle.full_attention(q, k, v)
    torch.testing.assert_close(got, exp.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("dtype,d,causal", [(torch.bfloat16, 64, False), (torch.float16, 128, True), (torch.bfloat16, 32, False)])
def test_fixed_block_16bit(pisa, dtype, d, causal):
    gen = torch.Generator().manual_seed(d)
    q, k, v = (torch.randn((1, 4, 200, d), generator=gen).to(dtype) for _ in range(3))
    got = pisa.fixed_block_attention(q.to(DEV), k.to(DEV), v.to(DEV), 1 / math.sqrt(d), causal).cpu().float()
    exp = oracle.fixed_block_attention(q, k, v, causal=causal, round_p=True).float()
    torch.testing.assert_close(got, exp, atol=2e-2, rtol=2e-2)


def test_fixed_block_fp32_config1(pisa):
    gen = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn((1, 8, 1024, 64), generator=gen) for _ in range(3))
    got = pisa.fixed_block_attention(q.to(DEV), k.to(DEV), v.to(DEV), 1 / 8.0).cpu()
    exp = oracle.fixed_block_attention(q, k, v)
    assert (got - exp).abs().max().item() <= 1e-4


@pytest.mark.parametrize("tokens,d,causal", [(200, 40, True), (1000, 128, False), (90, 64, True), (64, 8, False)])
def test_fixed_block_fp32_ragged_causal(pisa, tokens, d, causal):
    # T=200: the last block has 8 rows, so its second 32-row half is empty
    gen = torch.Generator().manual_seed(tokens + d)
    q, k, v = (torch.randn((2, 3, tokens, d), generator=gen) for _ in range(3))
    got = pisa.fixed_block_attention(q.to(DEV), k.to(DEV), v.to(DEV), d ** -0.5, causal).cpu()
    exp = oracle.fixed_block_attention(q, k, v, causal=causal)
    assert (got - exp).abs().max().item() <= 1e-4


def test_h3_pack_bit_exact(pisa):
    gen = torch.Generator().manual_seed(9170)
    qkv = torch.randn((1, 300, 3, 56, 128), generator=gen).to(torch.bfloat16).to(DEV)
    q = qkv[:, :, 0].permute(0, 2, 1, 3)
    k = qkv[:, :, 1].permute(0, 2, 1, 3)
    v = qkv[:, :, 2].permute(0, 2, 1, 3)
    packed = pisa.pack_views([q, k, v])
    for i, x in enumerate((q, k, v)):
        assert torch.equal(packed[i], x.contiguous())


def test_generic_forward_matches_oracle(pisa):
    (q, k, v), (qd, kd, vd) = _bh_inputs(2, 1000, 5)
    got = pisa.generic_forward(qd, kd, vd, exact_blocks=3, scale=1 / math.sqrt(128)).cpu().float()
    exp, _ = oracle.generic_forward(q, k, v, 3)
    torch.testing.assert_close(got, exp.float(), **TOL)
