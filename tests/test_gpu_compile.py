"""Outer torch.compile(fullgraph=True) through the custom ops, as the
reference tests its wheel (native/rdna35_pisa_ck/tests/test_forward.py:203-209):
the compiled graph calls the same native kernels and matches eager."""
import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV, to_dev_bhtd

pytestmark = pytest.mark.gpu


def _compile_target(q, k, v):
    import b200_pisa

    return b200_pisa.forward(q, k, v, exact_blocks=1)


def _spatial_target(q, k, v):
    import b200_pisa

    return b200_pisa.forward_spatial_bhtd(q, k, v, exact_blocks=23) * 2.0


def test_outer_torch_compile_fullgraph():
    import b200_pisa

    torch._dynamo.reset()
    gen = torch.Generator().manual_seed(31)
    q, k, v = (torch.randn((1, 64, 128), generator=gen).to(torch.bfloat16).to(DEV) for _ in range(3))
    b200_pisa.prepare()
    expected = _compile_target(q, k, v)
    compiled = torch.compile(_compile_target, backend="inductor", fullgraph=True)
    actual = compiled(q, k, v)
    torch.testing.assert_close(actual, expected, atol=1e-3, rtol=1e-3)


def test_outer_torch_compile_spatial_fullgraph():
    import b200_pisa

    torch._dynamo.reset()
    q, k, v = (to_dev_bhtd(x) for x in oracle.anima_inputs(batch=1, heads=2, seed=8))
    expected = _spatial_target(q, k, v)
    compiled = torch.compile(_spatial_target, backend="inductor", fullgraph=True)
    actual = compiled(q, k, v)
    assert b200_pisa.capabilities()["outer_torch_compile"]
    torch.testing.assert_close(actual, expected, atol=0, rtol=0)
