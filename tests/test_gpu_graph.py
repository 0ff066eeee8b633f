"""A whole PISA call captured in a CUDA graph and replayed: the kernels the
C ABI launches (statistics, reduction, centroid copies, routing, pairing,
attention, with programmatic dependent launch between them) record into the
capture stream, and each replay reproduces the eager output bit for bit on
new inputs copied into the captured buffers."""
import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV, to_dev_bhtd

pytestmark = pytest.mark.gpu


def test_forward_spatial_bhtd_replays_from_a_cuda_graph():
    import b200_pisa

    q, k, v = (to_dev_bhtd(x) for x in oracle.anima_inputs(batch=1, heads=4, seed=12))
    b200_pisa.forward_spatial_bhtd(q, k, v, exact_blocks=23)  # warm-up outside capture (attributes, caches)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            out = b200_pisa.forward_spatial_bhtd(q, k, v, exact_blocks=23)
    torch.cuda.synchronize()
    for seed in (13, 14):
        fresh = [to_dev_bhtd(x) for x in oracle.anima_inputs(batch=1, heads=4, seed=seed)]
        for dst, src in zip((q, k, v), fresh):
            dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        eager = b200_pisa.forward_spatial_bhtd(*fresh, exact_blocks=23)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
