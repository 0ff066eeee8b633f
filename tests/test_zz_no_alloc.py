"""GPU tests of the allocation-free statistics entry point.

b2_pisa_block_stats_noalloc serves callers that cannot allocate device memory
when they run (allocator callbacks, fixed memory pools, plugin hosts that only
hand out input and output buffers): its scratch is an array compiled into the
library.  Each case calls it twice in a row through the C ABI (the array keeps
the previous call's contents) and checks every output against the
workspace-based b2_pisa_block_stats: bit for bit while the block grouping is
the workspace entry's own, within FP32 reassociation where the 8 MiB array
forces larger groups.  The file is named so pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NAMES = ("qc", "kc", "vc", "hs", "hn", "h16")


def _bind():
    from b200_pisa import _lib

    lib = _lib.LIB
    lib.b2_pisa_block_stats_noalloc.restype = ctypes.c_int
    lib.b2_pisa_block_stats_noalloc.argtypes = [ctypes.POINTER(_lib.View)] * 3 + [ctypes.c_int32] + [ctypes.c_void_p] * 7
    return _lib, lib


def _outputs(bh, blocks, dtype, mode, dev):
    from b200_pisa import _lib

    cent = torch.float32 if mode == _lib.STATS_GENERIC else dtype
    return dict(
        qc=torch.full((bh, blocks, 128), float("nan"), device=dev, dtype=cent),
        kc=torch.full((bh, blocks, 128), float("nan"), device=dev, dtype=torch.float32),
        vc=torch.full((bh, blocks, 128), float("nan"), device=dev, dtype=cent),
        hs=torch.full((bh, 128, 128), float("nan"), device=dev, dtype=torch.float32),
        hn=torch.full((bh, blocks), float("nan"), device=dev, dtype=torch.float32),
        h16=torch.full((bh, 128, 128), float("nan"), device=dev, dtype=dtype),
    )


def _inputs(seed, batch, heads, tokens, dtype, tiled, dev):
    """q/k/v as BHTD views of raster [B,T,H,128] storage (tiled) or [BH,T,128]."""
    gen = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for _ in range(3):
        x = torch.randn((batch, tokens, heads, 128), device=dev, generator=gen)
        x = (x + 0.5 * torch.randn((batch, 1, heads, 128), device=dev, generator=gen)).to(dtype)
        out.append(x.permute(0, 2, 1, 3) if tiled else x.permute(0, 2, 1, 3).reshape(batch * heads, tokens, 128))
    return out


CASES = [
    # (dtype, mode, tiled grid or None, batch, heads, tokens)
    (torch.bfloat16, "HYD", None, 1, 32, 9216),  # groups grown to fit 8 MiB
    (torch.bfloat16, "HYD", (32, 48), 2, 3, 1536),
    (torch.float16, "HYD", None, 1, 4, 1000),
    (torch.bfloat16, "GENERIC", None, 1, 4, 4160),
    (torch.float16, "GENERIC", (16, 16), 2, 2, 512),
    (torch.bfloat16, "SCALED", None, 1, 3, 777),
    (torch.float16, "SCALED", (24, 16), 1, 2, 768),
]


@pytest.mark.parametrize("dtype,mode,grid,batch,heads,tokens", CASES)
def test_noalloc_stats_match_workspace_entry_point(dtype, mode, grid, batch, heads, tokens):
    _lib, lib = _bind()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    code = {"HYD": _lib.STATS_HYD, "GENERIC": _lib.STATS_GENERIC, "SCALED": _lib.STATS_SCALED}[mode]
    bh = batch * heads
    blocks = (tokens + 63) // 64
    # the workspace entry's grouping: 16 blocks per partial; grown when the array is too small
    grown = bh * ((blocks + 15) // 16) * 128 * 128 * 4 > (8 << 20)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed in (1, 2):  # two calls in a row share the scratch array
        q, k, v = _inputs(seed, batch, heads, tokens, dtype, grid is not None, dev)
        if grid is None:
            views = [_lib.view(x) for x in (q, k, v)]
        else:
            views = [_lib.view(x, order=_lib.ORDER_TILED8, grid=grid) for x in (q, k, v)]
        ref = _outputs(bh, blocks, dtype, code, dev)
        ws = torch.empty(int(lib.b2_stats_workspace_bytes(bh, tokens, 128)), device=dev, dtype=torch.uint8)
        _lib.check(lib.b2_pisa_block_stats(*(ctypes.byref(x) for x in views), code,
                                           *(ref[n].data_ptr() for n in NAMES), ws.data_ptr(), stream))
        got = _outputs(bh, blocks, dtype, code, dev)
        rc = lib.b2_pisa_block_stats_noalloc(*(ctypes.byref(x) for x in views), code,
                                             *(got[n].data_ptr() for n in NAMES), stream)
        assert rc == 0, lib.b2_last_error().decode()
        torch.cuda.synchronize()
        for n in ("qc", "kc", "vc"):
            torch.testing.assert_close(got[n], ref[n], atol=0, rtol=0)
        if code == _lib.STATS_HYD:
            torch.testing.assert_close(got["hn"], ref["hn"], atol=0 if not grown else 1e-2, rtol=0 if not grown else 1e-3)
        if grown:
            torch.testing.assert_close(got["hs"], ref["hs"], atol=2e-3, rtol=1e-4)
            torch.testing.assert_close(got["h16"].float(), ref["h16"].float(), atol=1e-2, rtol=1e-2)
        else:
            torch.testing.assert_close(got["hs"], ref["hs"], atol=0, rtol=0)
            torch.testing.assert_close(got["h16"], ref["h16"], atol=0, rtol=0)


def test_noalloc_rejects_oversized_request():
    _lib, lib = _bind()
    dev = torch.device("cuda", 0)
    x = torch.zeros((129, 64, 128), device=dev, dtype=torch.bfloat16)
    view = _lib.view(x)
    out = torch.empty(129 * 128 * 128, device=dev, dtype=torch.float32)
    rc = lib.b2_pisa_block_stats_noalloc(ctypes.byref(view), ctypes.byref(view), ctypes.byref(view), _lib.STATS_HYD,
                                         out.data_ptr(), out.data_ptr(), out.data_ptr(), out.data_ptr(), None, None,
                                         torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.B2_ERR_UNSUPPORTED
    assert "8 MiB" in lib.b2_last_error().decode()
