"""GPU checks of the tcgen05 attention pipeline's synchronisation.

The attention kernel hands TMEM buffers between the tensor core and the
softmax warps through mbarriers; a missing wait shows up as rare,
input-timing-dependent garbage (NaNs in a few columns, run-to-run
differences), most often when the running max keeps growing and O is
rescaled.  These tests run the largest grids with logit ranges that force
frequent rescaling, repeat each call, and require finite, bitwise-repeatable
outputs that match the oracle, with the kernel status word clear.
"""
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


def _repeat(fn, times=3):
    from b200_pisa import _lib

    outs = []
    for _ in range(times):
        outs.append(fn().clone())
        torch.cuda.synchronize()
        assert _lib.read_status() == 0, "a pipeline wait timed out"
    for o in outs[1:]:
        assert torch.equal(o, outs[0]), "outputs differ between identical calls"
    assert torch.isfinite(outs[0]).all()
    return outs[0]


def test_spatial_16_heads_wide_offsets(pisa):
    # per-tile offsets of sigma 2 give logits spread over tens of units:
    # the lazy running max is exceeded and O rescaled on many tiles
    q, k, v = oracle.anima_inputs(batch=1, heads=16, seed=9, offset_sigma=2.0)
    qd, kd, vd = (to_dev_bhtd(x) for x in (q, k, v))
    got = _repeat(lambda: pisa.forward_spatial_bhtd(qd, kd, vd, exact_blocks=23)).cpu().float()
    exp, _ = oracle.hyd_forward_spatial(q[:, :4], k[:, :4], v[:, :4], 23)
    torch.testing.assert_close(got[:, :, : 4 * 128], exp.float(), **TOL)


def test_linear_32_heads_repeatable(pisa):
    # the benchmark's grid size (2304 CTAs) on contiguous [BH, T, 128] inputs
    q, k, v = oracle.generic_inputs(32, 9216, 21)
    qd, kd, vd = (x.to(DEV) for x in (q, k, v))
    got = _repeat(lambda: pisa.forward(qd, kd, vd, exact_blocks=23)).cpu().float()
    exp, _ = oracle.hyd_forward(q[:2], k[:2], v[:2], 23)
    torch.testing.assert_close(got[:2], exp.float(), **TOL)


def test_dense_large_logits_match_sdpa(pisa):
    # scaled q: logits up to ~50 in the log2 domain, rescales on most tiles
    gen = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn((1, 4, 4096, 128), generator=gen) for _ in range(3))
    q = q * 6.0
    qd, kd, vd = (x.to(DEV, torch.bfloat16) for x in (q, k, v))
    got = _repeat(lambda: pisa.full_attention(qd, kd, vd, 128 ** -0.5)).float()
    exp = F.scaled_dot_product_attention(qd.float(), kd.float(), vd.float(), scale=128 ** -0.5)
    torch.testing.assert_close(got, exp, atol=2e-2, rtol=2e-2)


def _greedy_pairs(sel):
    """Restatement of pair_kernel: blocks in ascending order; each unpaired
    block takes the later unpaired block of largest selection overlap (ties:
    lowest index), or stays single when none is left."""
    nb = sel.shape[0]
    ov = (sel[:, None, :] & sel[None, :, :]).sum(-1)
    used = [False] * nb
    pairs = []
    for a in range(nb):
        if used[a]:
            continue
        used[a] = True
        cands = [(int(ov[a, j]), -j) for j in range(a + 1, nb) if not used[j]]
        b = -max(cands)[1] if cands else -1
        if b >= 0:
            used[b] = True
        pairs.append((a, b))
    return pairs


@pytest.mark.parametrize("blocks", [7, 144, 300, 512, 608])
def test_pairing_kernel_matches_restatement(pisa, blocks):
    import ctypes

    from b200_pisa import LIB, check

    gen = torch.Generator().manual_seed(blocks)
    bh, words = 3, (blocks + 31) // 32
    sel = torch.rand((bh, blocks, blocks), generator=gen) < 0.2
    packed = torch.zeros((bh, blocks, words), dtype=torch.int64)
    for w in range(words):
        chunk = sel[:, :, 32 * w: 32 * w + 32].to(torch.int64)
        packed[:, :, w] = (chunk << torch.arange(chunk.shape[-1], dtype=torch.int64)).sum(-1)
    packed = packed.to(torch.int32).to(DEV)  # two's complement bit pattern of the uint32 words
    npairs = (blocks + 1) // 2
    out = torch.full((bh, npairs, 2), -7, dtype=torch.int32, device=DEV)
    check(LIB.b2_pisa_pair(ctypes.c_void_p(packed.data_ptr()), bh, blocks, ctypes.c_void_p(out.data_ptr()),
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    got = out.cpu()
    for b in range(bh):
        exp = _greedy_pairs(sel[b].numpy())
        assert [tuple(p) for p in got[b].tolist()] == exp
        seen = sorted(x for p in exp for x in p if x >= 0)
        assert seen == list(range(blocks))


def test_spatial_batch_two_matches_oracle(pisa):
    # the benchmark's batch of 2: the 8x8-tiled maps address frame * batch
    q, k, v = oracle.anima_inputs(batch=2, heads=2, seed=13)
    qd, kd, vd = (to_dev_bhtd(x) for x in (q, k, v))
    got = _repeat(lambda: pisa.forward_spatial_bhtd(qd, kd, vd, exact_blocks=23)).cpu().float()
    exp, _ = oracle.hyd_forward_spatial(q, k, v, 23)
    assert got.shape == (2, 9216, 256)
    torch.testing.assert_close(got, exp.float(), **TOL)


@pytest.mark.parametrize("heads_per_stage", [1, 2, 4])
def test_host_pipelined_forward_equals_device_forward(pisa, heads_per_stage):
    # staged copies + per-stage forwards give the same bits as one device call
    q, k, v = oracle.anima_inputs(batch=2, heads=4, seed=17)
    host = [x.permute(0, 2, 1, 3).contiguous().pin_memory().permute(0, 2, 1, 3) for x in (q, k, v)]
    dev = [to_dev_bhtd(x) for x in (q, k, v)]
    exp = pisa.forward_spatial_bhtd(*dev, exact_blocks=23).cpu()
    out = pisa.forward_spatial_bhtd_host(*host, exact_blocks=23, heads_per_stage=heads_per_stage)
    torch.cuda.synchronize()
    assert out.shape == (2, 9216, 512) and out.is_pinned()
    assert torch.equal(out, exp)
    # and again into the same pinned output, as a sampling loop would
    out.zero_()
    pisa.forward_spatial_bhtd_host(*host, exact_blocks=23, heads_per_stage=heads_per_stage, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, exp)


def test_host_pipelined_forward_rejects_pageable_inputs(pisa):
    q, k, v = oracle.anima_inputs(batch=1, heads=2, seed=1)
    with pytest.raises(ValueError, match="pinned"):
        pisa.forward_spatial_bhtd_host(q, k, v, exact_blocks=23)


def test_output_of_a_head_does_not_depend_on_the_other_heads(pisa):
    # statistics group blocks by the block count only, so a head computed
    # alone or with others (sharded, staged) gives the same bits
    q, k, v = oracle.generic_inputs(6, 9216, 23)
    qd, kd, vd = (x.to(DEV) for x in (q, k, v))
    full = pisa.forward(qd, kd, vd, exact_blocks=23)
    part = pisa.forward(qd[2:4].contiguous(), kd[2:4].contiguous(), vd[2:4].contiguous(), exact_blocks=23)
    one = pisa.forward(qd[5:6].contiguous(), kd[5:6].contiguous(), vd[5:6].contiguous(), exact_blocks=23)
    assert torch.equal(part, full[2:4])
    assert torch.equal(one, full[5:6])


def test_host_pipelined_forward_from_two_threads(pisa):
    # the per-device copy streams and events are shared: concurrent calls
    # from two host threads (each on its own compute stream) stay correct
    import threading

    q, k, v = oracle.anima_inputs(batch=1, heads=4, seed=29)
    host = [x.permute(0, 2, 1, 3).contiguous().pin_memory().permute(0, 2, 1, 3) for x in (q, k, v)]
    exp = pisa.forward_spatial_bhtd(*(to_dev_bhtd(x) for x in (q, k, v)), exact_blocks=23).cpu()
    outs, errors = [None, None], []

    def worker(i):
        try:
            stream = torch.cuda.Stream(DEV)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    outs[i] = pisa.forward_spatial_bhtd_host(*host, exact_blocks=23, heads_per_stage=1)
                stream.synchronize()
        except Exception as exc:  # reported below
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for out in outs:
        assert torch.equal(out, exp)
