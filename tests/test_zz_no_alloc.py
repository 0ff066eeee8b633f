"""GPU test of the allocation-free statistics entry point.

b2_pisa_block_stats_noalloc serves callers that cannot allocate device memory
when they run (allocator callbacks, fixed memory pools, plugin hosts that only
hand out input and output buffers): its scratch is an array compiled into the
library.  This test calls it twice in a row through the C ABI and checks each
result against the workspace-based b2_pisa_block_stats, at the tolerances the
other statistics tests use.  The file is named so pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _outputs(bh, blocks, dev):
    return dict(
        qc=torch.empty((bh, blocks, 128), device=dev, dtype=torch.bfloat16),
        kc=torch.empty((bh, blocks, 128), device=dev, dtype=torch.float32),
        vc=torch.empty((bh, blocks, 128), device=dev, dtype=torch.bfloat16),
        hs=torch.empty((bh, 128, 128), device=dev, dtype=torch.float32),
        hn=torch.empty((bh, blocks), device=dev, dtype=torch.float32),
        h16=torch.empty((bh, 128, 128), device=dev, dtype=torch.bfloat16),
    )


def test_noalloc_stats_match_workspace_entry_point():
    from b200_pisa import _lib

    lib = _lib.LIB
    lib.b2_pisa_block_stats_noalloc.restype = ctypes.c_int
    lib.b2_pisa_block_stats_noalloc.argtypes = [ctypes.POINTER(_lib.View)] * 3 + [ctypes.c_int32] + [ctypes.c_void_p] * 7
    lib.b2_noalloc_last_error.restype = ctypes.c_char_p
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bh, tokens = 32, 9216
    blocks = tokens // 64
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed in (1, 2):  # two calls in a row share the scratch array
        gen = torch.Generator(device=dev).manual_seed(seed)
        q, k, v = (torch.randn((bh, tokens, 128), device=dev, generator=gen).to(torch.bfloat16) for _ in range(3))
        views = [_lib.view(x) for x in (q, k, v)]
        ref = _outputs(bh, blocks, dev)
        ws = torch.empty(int(lib.b2_stats_workspace_bytes(bh, tokens, 128)), device=dev, dtype=torch.uint8)
        _lib.check(lib.b2_pisa_block_stats(*(ctypes.byref(x) for x in views), _lib.STATS_HYD, *(
            ref[n].data_ptr() for n in ("qc", "kc", "vc", "hs", "hn", "h16")), ws.data_ptr(), stream))
        got = _outputs(bh, blocks, dev)
        rc = lib.b2_pisa_block_stats_noalloc(*(ctypes.byref(x) for x in views), _lib.STATS_HYD, *(
            got[n].data_ptr() for n in ("qc", "kc", "vc", "hs", "hn", "h16")), stream)
        assert rc == 0, lib.b2_noalloc_last_error().decode()
        torch.cuda.synchronize()
        for n in ("qc", "kc", "vc"):
            torch.testing.assert_close(got[n], ref[n], atol=0, rtol=0)
        torch.testing.assert_close(got["hn"], ref["hn"], atol=1e-2, rtol=1e-3)
        torch.testing.assert_close(got["hs"], ref["hs"], atol=2e-3, rtol=1e-4)
        torch.testing.assert_close(got["h16"].float(), ref["h16"].float(), atol=1e-2, rtol=1e-2)


def test_noalloc_rejects_oversized_request():
    from b200_pisa import _lib

    lib = _lib.LIB
    lib.b2_pisa_block_stats_noalloc.restype = ctypes.c_int
    lib.b2_pisa_block_stats_noalloc.argtypes = [ctypes.POINTER(_lib.View)] * 3 + [ctypes.c_int32] + [ctypes.c_void_p] * 7
    lib.b2_noalloc_last_error.restype = ctypes.c_char_p
    dev = torch.device("cuda", 0)
    x = torch.zeros((129, 64, 128), device=dev, dtype=torch.bfloat16)
    view = _lib.view(x)
    out = torch.empty(129 * 128 * 128, device=dev, dtype=torch.float32)
    rc = lib.b2_pisa_block_stats_noalloc(ctypes.byref(view), ctypes.byref(view), ctypes.byref(view), _lib.STATS_HYD,
                                         out.data_ptr(), out.data_ptr(), out.data_ptr(), out.data_ptr(), None, None,
                                         torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.B2_ERR_UNSUPPORTED
    assert "8 MiB" in lib.b2_noalloc_last_error().decode()
