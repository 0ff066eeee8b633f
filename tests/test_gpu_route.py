"""GPU routing (centroid scores + per-query-block top-k) against the oracle.

The selected key-block index sets must equal the oracle's
(topk(k).indices.sort(), rdna35_pisa_ck/__init__.py:258-269 for HYD,
generic_pisa.py:172-184 for the generic path) on every row except those the
oracle flags as score near-ties (k-th and (k+1)-th scores within 1e-5
relative), where FP32 summation order may legitimately swap the cut.  The
selection bitsets must agree with the index lists on every row.
"""
import ctypes
import math

import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV

pytestmark = pytest.mark.gpu


def _route(qc, kc, h_norm, k, scale, *, hyd, sink=-2):
    from b200_pisa import LIB, _lib, check

    bh, nb, d = qc.shape
    words = (nb + 31) // 32
    qd = qc.to(DEV, torch.bfloat16 if hyd else torch.float32).contiguous()
    kd = kc.to(DEV, torch.float32).contiguous()
    hd = h_norm.to(DEV, torch.float32).contiguous() if h_norm is not None else None
    idx = torch.full((bh, nb, max(k, 1)), -7, dtype=torch.int32, device=DEV)
    sel = torch.full((bh, nb, words), -1, dtype=torch.int32, device=DEV)
    code = _lib.B2_BF16 if hyd else _lib.B2_F32
    check(LIB.b2_pisa_route(qd.data_ptr(), code, kd.data_ptr(), code, hd.data_ptr() if hd is not None else None,
                            bh, nb, d, k, scale, sink, idx.data_ptr(), sel.data_ptr(),
                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    return idx.cpu().long()[..., :k], sel.cpu()


def _unpack(sel, nb):
    words = sel.to(torch.int64) & 0xFFFFFFFF
    bits = (words[..., :, None] >> torch.arange(32)) & 1
    return bits.flatten(-2)[..., :nb].bool()


def _check(idx, sel, exp, scores, k, nb):
    ties = oracle.near_tie_rows(scores, k)
    clean = ~ties
    assert clean.float().mean() > 0.9, "too many near-tie rows for a meaningful check"
    assert torch.equal(idx[clean], exp[clean])
    # bitsets and lists agree everywhere (also on near-tie rows)
    from_idx = torch.zeros(idx.shape[:-1] + (nb,), dtype=torch.bool)
    from_idx.scatter_(-1, idx, True)
    assert torch.equal(_unpack(sel, nb), from_idx)
    assert (idx.diff(dim=-1) > 0).all(), "indices must be strictly ascending"


def _centroids(bh, nb, seed, d=128):
    gen = torch.Generator().manual_seed(seed)
    base = torch.randn((bh, 1, d), generator=gen)
    qc = base + 0.7 * torch.randn((bh, nb, d), generator=gen)
    kc = base + 0.7 * torch.randn((bh, nb, d), generator=gen)
    hn = torch.rand((bh, nb), generator=gen) * 50 + 1
    return qc, kc, hn


@pytest.mark.parametrize("nb,k,sink", [(144, 23, None), (144, 23, 0), (144, 23, -1), (37, 5, None), (600, 100, None)])
def test_hyd_route_matches_oracle(nb, k, sink):
    qc, kc, hn = _centroids(3, nb, nb + k)
    scale = 128 ** -0.5
    idx, sel = _route(qc, kc, hn, k, scale, hyd=True, sink=-2 if sink is None else sink)
    scores = oracle.route_scores_hyd(qc.to(torch.bfloat16), kc, hn, scale)
    exp = oracle.select_topk(scores, k, None if sink is None else (sink % nb))
    if sink is not None:
        scores = scores.clone()
        scores[..., sink % nb] = torch.inf
    _check(idx, sel, exp, scores, k, nb)


@pytest.mark.parametrize("nb,k", [(512, 86), (1000, 7), (1024, 1000), (33, 1)])
def test_generic_route_matches_oracle(nb, k):
    qc, kc, _ = _centroids(2, nb, 3 * nb + k)
    scale = 128 ** -0.5
    idx, sel = _route(qc, kc, None, k, scale, hyd=False)
    scores = oracle.route_scores_generic(qc, kc, scale)
    _check(idx, sel, oracle.select_topk(scores, k), scores, k, nb)


@pytest.mark.parametrize("nb,k", [(300, 40), (64, 64), (1024, 3)])
def test_route_all_ties_take_lowest_indices(nb, k):
    # zero query centroids: every score ties, so the k lowest block indices win
    qc = torch.zeros((2, nb, 128))
    kc = torch.randn((2, nb, 128), generator=torch.Generator().manual_seed(nb))
    for hyd in (True, False):
        hn = torch.ones((2, nb)) if hyd else None
        idx, sel = _route(qc, kc, hn, k, 128 ** -0.5, hyd=hyd)
        assert torch.equal(idx, torch.arange(k).expand(2, nb, k))
        assert _unpack(sel, nb).sum(-1).eq(k).all()


def test_route_from_anima_statistics():
    # routing fed by the oracle's HYD statistics of config-3 style inputs
    q, k, v = oracle.anima_inputs(batch=1, heads=2, seed=3)
    packed = [oracle.pack_spatial(x) for x in (q, k, v)]
    qc, kc, _, _, hn = oracle.hyd_block_stats(*packed)
    scale = float(torch.tensor(1 / math.sqrt(128), dtype=torch.float32))
    idx, sel = _route(qc, kc, hn, 23, scale, hyd=True)
    scores = oracle.route_scores_hyd(qc, kc, hn, scale)
    _check(idx, sel, oracle.select_topk(scores, 23), scores, 23, 144)
