"""GPU parity at the BASELINE configurations' own shapes.

* Config 3 (Anima PISA, B=2 H=16 T=9216, 23/144 exact): the index sets the
  GPU pipeline routes to (GPU statistics -> GPU routing, read back from the
  call's workspace) against the oracle's
  select_topk(route_scores_hyd(hyd_block_stats(...))) on every
  (batch, head, query block), and the whole output against the oracle.
  Rows may differ only on documented near-ties: the k-th and (k+1)-th oracle
  scores lie within 1e-5*max(1,|s|) plus twice the bound on the GPU's
  per-column score error (its measured max |d log(h_norm + 1e-5)| plus the
  FP32 dot-product error bound n*u*sum|qc*kc|*scale).
* Config 2: exact full self-attention at T=9216 and cross-attention against
  512 keys, B=2 H=16; sampled heads against the oracle.
* Config 4: MiniMax-H3 exact attention on the interleaved [1,T,3,56,128]
  projection views at T=9170 (KV profile) and T=16500 (QKV profile); sampled
  heads against the oracle, the pack bit-exact.
* Config 5: generic PISA at T=32760, H=40, 86 of 512 exact blocks; index
  sets and sampled heads' outputs against the oracle.
The oracle runs on sampled heads only (every (batch, head) is independent).
"""
import math

import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV, to_dev_bhtd

pytestmark = pytest.mark.gpu

TOL = dict(atol=5e-2, rtol=5e-2)  # BF16 gate of native/rdna35_pisa_ck/tests/test_forward.py:113-117
EXACT_TOL = dict(atol=2e-2, rtol=2e-2)


@pytest.fixture(scope="module")
def pisa():
    import b200_pisa

    b200_pisa.prepare()
    return b200_pisa


def _oracle_attention(q, k, v, scale, rows=2048):
    """Exact FP32 attention of one head [T,D] in query chunks (bounded memory)."""
    out = torch.empty((q.shape[0], v.shape[1]), dtype=torch.float32)
    kf, vf = k.float(), v.float()
    for s in range(0, q.shape[0], rows):
        o, _ = oracle._softmax_attend(q[s:s + rows].float(), kf, vf, scale)
        out[s:s + rows] = o
    return out


def _score_error_bound(qc, kc, scale):
    """FP32 accumulation bound of the D=128 routing dot products."""
    mag = torch.bmm(qc.float().abs(), kc.float().abs().transpose(1, 2)).max().item()
    return 128 * 2.0 ** -24 * mag * scale


def test_config3_index_sets_and_output_end_to_end(pisa):
    q, k, v = oracle.anima_inputs(batch=2, heads=16, seed=5)
    out, idx, h_norm = pisa.forward_spatial_bhtd_with_routing(*(to_dev_bhtd(x) for x in (q, k, v)), exact_blocks=23)
    torch.cuda.synchronize()
    idx, h_norm, out = idx.cpu().long(), h_norm.cpu(), out.cpu()
    packed = [oracle.pack_spatial(x) for x in (q, k, v)]
    stats = oracle.hyd_block_stats(*packed)
    qc, kc, _, _, hn_ref = stats
    scale = float(torch.tensor(1.0 / math.sqrt(128), dtype=torch.float32))
    scores = oracle.route_scores_hyd(qc, kc, hn_ref, scale)
    ref_idx = oracle.select_topk(scores, 23)
    assert idx.shape == ref_idx.shape == (32, 144, 23)
    assert torch.all(idx[..., 1:] > idx[..., :-1]), "indices must be ascending and distinct"
    d_log = (torch.log(h_norm + 1e-5) - torch.log(hn_ref + 1e-5)).abs().max().item()
    abs_tol = 2 * (d_log + _score_error_bound(qc, kc, scale))
    ties = oracle.near_tie_rows(scores, 23, abs_tol=abs_tol)
    mismatched = (idx != ref_idx).any(-1)
    outside = mismatched & ~ties
    print(f"config 3 routing: {int(mismatched.sum())} of {mismatched.numel()} rows differ, "
          f"{int(ties.sum())} near-tie rows (window {abs_tol:.3g}, max |d log h_norm| {d_log:.3g}), "
          f"{int(outside.sum())} differ outside the window")
    assert int(outside.sum()) == 0
    assert d_log < 1e-3
    exp, _ = oracle.hyd_forward_batched(*packed, 23, stats=stats)
    exp = oracle.unpack_spatial(exp, 2, 16)
    torch.testing.assert_close(out.float(), exp.float(), **TOL)


def test_config2_full_self_attention_t9216(pisa):
    gen = torch.Generator().manual_seed(9216)
    q, k, v = (torch.randn((2, 16, 9216, 128), generator=gen).to(torch.bfloat16) for _ in range(3))
    out = pisa.full_attention(q.to(DEV), k.to(DEV), v.to(DEV), 1.0 / math.sqrt(128)).cpu()
    for b, h in ((0, 0), (1, 15)):
        exp = _oracle_attention(q[b, h], k[b, h], v[b, h], 1.0 / math.sqrt(128))
        torch.testing.assert_close(out[b, h].float(), exp, **EXACT_TOL)


def test_config2_cross_attention_512_keys(pisa):
    gen = torch.Generator().manual_seed(512)
    q = torch.randn((2, 16, 9216, 128), generator=gen).to(torch.bfloat16)
    k, v = (torch.randn((2, 16, 512, 128), generator=gen).to(torch.bfloat16) for _ in range(2))
    out = pisa.full_attention(q.to(DEV), k.to(DEV), v.to(DEV), 1.0 / math.sqrt(128)).cpu()
    for b, h in ((0, 3), (1, 12)):
        exp = _oracle_attention(q[b, h], k[b, h], v[b, h], 1.0 / math.sqrt(128))
        torch.testing.assert_close(out[b, h].float(), exp, **EXACT_TOL)


@pytest.mark.parametrize("tokens,profile", [(9170, "kv"), (16500, "qkv")])
def test_config4_minimax_h3_full_shape(tokens, profile):
    from rdna35_block_attention.minimax_h3_gfx1151_attention import (
        make_minimax_h3_gfx1151_attention_override, minimax_h3_pack_profile, pack_minimax_h3_qkv)

    assert minimax_h3_pack_profile(tokens) == profile
    gen = torch.Generator().manual_seed(tokens)
    qkv = torch.randn((1, tokens, 3, 56, 128), generator=gen).to(torch.bfloat16)
    dv = qkv.to(DEV)
    views = [dv[:, :, i].permute(0, 2, 1, 3) for i in range(3)]

    def original(*args, **kwargs):
        raise AssertionError("the eligible H3 call must not chain to the previous backend")

    override = make_minimax_h3_gfx1151_attention_override(device_index=0, verbose_fallbacks=False,
                                                          previous_override=None)
    out = override(original, *views, 56, skip_reshape=True).cpu()
    assert out.shape == (1, tokens, 56 * 128)
    out = out.view(1, tokens, 56, 128)
    for h in (0, 55):
        exp = _oracle_attention(qkv[0, :, 0, h], qkv[0, :, 1, h], qkv[0, :, 2, h], 1.0 / math.sqrt(128))
        torch.testing.assert_close(out[0, :, h].float(), exp, **EXACT_TOL)
    pq, pk, pv, got_profile = pack_minimax_h3_qkv(*views)
    assert got_profile == profile
    for packed, i in ((pq, 0), (pk, 1), (pv, 2)):
        assert torch.equal(packed, views[i])
    if profile == "qkv":
        assert pk.data_ptr() - pq.data_ptr() == pq.numel() * 2
    else:
        assert pv.data_ptr() - pk.data_ptr() == pk.numel() * 2


def test_config5_generic_pisa_video_full_shape(pisa):
    heads, tokens, exact = 40, 32760, 86
    q, k, v = oracle.generic_inputs(heads, tokens, seed=32760)
    scale = 1.0 / math.sqrt(128)
    out, idx = pisa.generic_forward(q.to(DEV), k.to(DEV), v.to(DEV), exact, scale, return_indices=True)
    out, idx = out.cpu(), idx.cpu().long()
    assert idx.shape == (heads, 512, exact)
    sample = [0, 39]
    qs, ks, vs = (x[sample] for x in (q, k, v))
    qc, kc, _, _, _ = oracle.generic_block_stats(qs, ks, vs)
    scores = oracle.route_scores_generic(qc, kc, scale)
    ref_idx = oracle.select_topk(scores, exact)
    # FP32 centroid sums in another order: ~1e-6 relative per centroid
    abs_tol = 2 * (_score_error_bound(qc, kc, scale) + 1e-5)
    ties = oracle.near_tie_rows(scores, exact, abs_tol=abs_tol)
    mismatched = (idx[sample] != ref_idx).any(-1)
    print(f"config 5 routing (heads {sample}): {int(mismatched.sum())} of {mismatched.numel()} rows differ, "
          f"{int(ties.sum())} near-tie rows, {int((mismatched & ~ties).sum())} outside the window")
    assert int((mismatched & ~ties).sum()) == 0
    exp, _ = oracle.generic_forward_batched(qs, ks, vs, exact, scale)
    torch.testing.assert_close(out[sample].float(), exp.float(), **TOL)


@pytest.mark.parametrize("sink", [0, -1])
def test_config3_sink_block_index_sets_and_output(pisa, sink):
    """The forced sink block (first or last key block always exact) at the
    full Anima size: routed sets contain the sink on every row and match the
    oracle's outside the near-tie window; outputs within the BF16 gate."""
    q, k, v = oracle.anima_inputs(batch=1, heads=4, seed=40 + sink)
    out, idx, h_norm = pisa.forward_spatial_bhtd_with_routing(*(to_dev_bhtd(x) for x in (q, k, v)), exact_blocks=23,
                                                              sink_block=sink)
    torch.cuda.synchronize()
    idx, h_norm, out = idx.cpu().long(), h_norm.cpu(), out.cpu()
    packed = [oracle.pack_spatial(x) for x in (q, k, v)]
    stats = oracle.hyd_block_stats(*packed)
    qc, kc, _, _, hn_ref = stats
    scale = float(torch.tensor(1.0 / math.sqrt(128), dtype=torch.float32))
    scores = oracle.route_scores_hyd(qc, kc, hn_ref, scale)
    ref_idx = oracle.select_topk(scores, 23, sink_block=sink)
    sink_index = 143 if sink == -1 else 0
    assert bool((idx == sink_index).any(-1).all())
    forced = scores.clone()
    forced[..., sink_index] = torch.inf
    d_log = (torch.log(h_norm + 1e-5) - torch.log(hn_ref + 1e-5)).abs().max().item()
    ties = oracle.near_tie_rows(forced, 23, abs_tol=2 * (d_log + _score_error_bound(qc, kc, scale)))
    assert int(((idx != ref_idx).any(-1) & ~ties).sum()) == 0
    exp, _ = oracle.hyd_forward_batched(*packed, 23, sink_block=sink, stats=stats)
    torch.testing.assert_close(out.float(), oracle.unpack_spatial(exp, 1, 4).float(), **TOL)
