"""Head sharding on one GPU: the shards of a 4-way split, computed as
separate calls and assembled by the interleave kernel of the all-gather
path, reproduce the single call bit for bit (config-3 shape, B=2 H=16)."""
import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_heads_reassemble_the_single_gpu_output(world):
    import b200_pisa
    from b200_pisa.sharded import head_range, interleave_shards

    q, k, v = oracle.anima_inputs(batch=2, heads=16, seed=21)
    raster = [x.permute(0, 2, 1, 3).contiguous().to(DEV) for x in (q, k, v)]  # [B,T,H,D]
    full = b200_pisa.forward_spatial_bhtd(*(x.permute(0, 2, 1, 3) for x in raster), exact_blocks=23)
    shards = []
    for rank in range(world):
        h0, h1 = head_range(16, world, rank)
        local = [x[:, :, h0:h1].contiguous().permute(0, 2, 1, 3) for x in raster]
        shards.append(b200_pisa.forward_spatial_bhtd(*local, exact_blocks=23))
    got = interleave_shards(torch.stack(shards))
    assert torch.equal(got, full)
