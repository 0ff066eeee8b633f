"""Masked fixed 64-token block attention on the B200 kernels.

Boolean and additive float masks in every rank form the reference accepts
(rdna35_block_attention/reference.py:114-156) run natively: the dispatcher
packs the masks' diagonal blocks into FP32 score terms on the device and the
tcgen05 (D=128, 16-bit), warp-MMA (D=32/64, 16-bit) and FP32 kernels add
them.  Outputs are checked against the oracle with the mask broadcast to
[B,H,T,T]: FP32 within the 1e-4 gate, 16-bit within 2e-2 (P rounded to the
input type as the kernels do), and fully masked rows NaN exactly where the
reference's softmax gives NaN."""
import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV

pytestmark = pytest.mark.gpu

B, H, T = 2, 3, 200


def _mask(kind, seed):
    gen = torch.Generator().manual_seed(seed)
    shapes = {"2d": (T, T), "3d_batch": (B, T, T), "3d_bh": (B * H, T, T), "4d_head": (1, H, T, T),
              "4d_full": (B, H, T, T)}
    shape = shapes[kind.split(":")[0]]
    if kind.endswith(":float"):
        return torch.randn(shape, generator=gen)
    mask = torch.rand(shape, generator=gen) > 0.3
    mask[..., 5, :] = False  # a fully masked query row in every (batch, head)
    return mask


def _broadcast(mask):
    """[B,H,T,T] form of a mask under the reference's rank rules."""
    if mask.ndim == 2:
        return mask.expand(B, H, T, T)
    if mask.ndim == 3 and mask.shape[0] == B:
        return mask[:, None].expand(B, H, T, T)
    if mask.ndim == 3:
        return mask.view(B, H, T, T)
    return mask.expand(B, H, T, T)


@pytest.mark.parametrize("dtype,dim", [(torch.float32, 64), (torch.float32, 128), (torch.bfloat16, 128),
                                       (torch.float16, 64), (torch.bfloat16, 32)])
@pytest.mark.parametrize("kind", ["2d", "3d_batch", "3d_bh:float", "4d_head", "4d_full:float"])
@pytest.mark.parametrize("causal", [False, True])
def test_native_masked_fixed_block_matches_oracle(dtype, dim, kind, causal):
    from rdna35_block_attention.dispatch import fixed_block_attention

    gen = torch.Generator().manual_seed(dim + T)
    q, k, v = (torch.randn((B, H, T, dim), generator=gen).to(dtype) for _ in range(3))
    mask = _mask(kind, dim)
    out, info = fixed_block_attention(q.to(DEV), k.to(DEV), v.to(DEV), layout="bhtd", causal=causal,
                                      mask=mask.to(DEV), return_diagnostics=True)
    assert info["backend"] == "b200", info
    exp = oracle.fixed_block_attention(q, k, v, causal=causal, mask=_broadcast(mask),
                                       round_p=dtype != torch.float32)
    got = out.cpu().float()
    assert torch.equal(torch.isnan(got), torch.isnan(exp)), "fully masked rows must be NaN, others finite"
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(got.nan_to_num(), exp.float().nan_to_num(), atol=tol, rtol=tol)


@pytest.mark.parametrize("layout", ["bthd", "bh_t_d"])
def test_masked_dispatch_in_other_layouts(layout):
    from rdna35_block_attention.dispatch import fixed_block_attention

    gen = torch.Generator().manual_seed(7)
    base = [torch.randn((B, H, T, 128), generator=gen).to(torch.bfloat16) for _ in range(3)]
    mask = _mask("2d", 3)
    if layout == "bthd":
        qkv = [x.permute(0, 2, 1, 3).reshape(B, T, H * 128) for x in base]
        kw = {"heads": H}
    else:
        qkv = [x.reshape(B * H, T, 128) for x in base]
        kw = {}
    out, info = fixed_block_attention(*(x.to(DEV) for x in qkv), layout=layout, mask=mask.to(DEV),
                                      return_diagnostics=True, **kw)
    assert info["backend"] == "b200", info
    exp = oracle.fixed_block_attention(*base, mask=_broadcast(mask), round_p=True)
    if layout == "bthd":
        exp = exp.permute(0, 2, 1, 3).reshape(B, T, H * 128)
    else:
        exp = exp.reshape(B * H, T, 128)
    got = out.cpu().float()
    assert torch.equal(torch.isnan(got), torch.isnan(exp))
    torch.testing.assert_close(got.nan_to_num(), exp.float().nan_to_num(), atol=2e-2, rtol=2e-2)
