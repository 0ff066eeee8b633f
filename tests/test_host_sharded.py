"""Head sharding of the PISA call over ranks, on CPU with two gloo ranks:
head ranges, the all-gather of per-rank [B,T,Hs*D] outputs and their
interleaving into the [B,T,H*D] raster (the exchange step of
b200_pisa.sharded; the attention itself needs the GPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_ranges_cover_every_head_once():
    from b200_pisa.sharded import head_range

    for heads, world in ((16, 1), (16, 2), (16, 4), (16, 8), (40, 8), (56, 8)):
        ranges = [head_range(heads, world, r) for r in range(world)]
        covered = [h for a, b in ranges for h in range(a, b)]
        assert covered == list(range(heads))
    with pytest.raises(ValueError):
        head_range(16, 3, 0)
    with pytest.raises(ValueError):
        head_range(16, 2, 2)


def test_interleave_matches_the_raster_layout():
    from b200_pisa.sharded import interleave_shards

    world, batch, tokens, width = 4, 2, 5, 8
    full = torch.arange(batch * tokens * world * width, dtype=torch.float32).view(batch, tokens, world * width)
    shards = torch.stack([full[..., n * width:(n + 1) * width] for n in range(world)])
    assert torch.equal(interleave_shards(shards), full)


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from b200_pisa.sharded import gather_head_shards, head_range

        batch, heads, tokens, dim = 2, 4, 6, 8
        gen = torch.Generator().manual_seed(0)  # every rank holds the same full call
        full = torch.randn((batch, tokens, heads, dim), generator=gen)
        h0, h1 = head_range(heads, world, rank)
        local = full[:, :, h0:h1].reshape(batch, tokens, (h1 - h0) * dim)  # "attention" = identity per head
        got = gather_head_shards(local)
        results[rank] = bool(torch.equal(got, full.reshape(batch, tokens, heads * dim)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_head_shards():
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    assert dict(results) == {0: True, 1: True}
