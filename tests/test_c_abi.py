"""The in-tree C-ABI library loads without a GPU and exports every entry
point include/b200attn.h declares; the ctypes table matches the header."""
import ctypes
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200attn.h"


def declared_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    from b200_pisa import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 15
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_covers_the_header():
    from b200_pisa import _lib

    names = declared_functions()
    # the allocation-free statistics entry point is bound by its own callers
    unbound = names - set(_lib.SIGNATURES) - {"b2_pisa_block_stats_noalloc", "b2_noalloc_last_error"}
    assert not unbound, unbound


def test_host_side_calls_without_gpu():
    from b200_pisa import _lib

    assert _lib.LIB.b2_api_version() == 7
    assert "architecture=sm_100a" in _lib.build_info_string()
    assert _lib.LIB.b2_pisa_workspace_bytes(32, 9216, 128, 23) > 0
    assert _lib.LIB.b2_pisa_workspace_bytes(32, 9216, 64, 23) == -1
    # no CUDA driver here: the device check fails with a CUDA error, not a crash
    assert _lib.LIB.b2_check_device(0) in (_lib.B2_ERR_CUDA, _lib.B2_ERR_DEVICE)
    assert _lib.LIB.b2_last_error()


def test_invalid_views_are_rejected_before_any_launch():
    import torch
    from b200_pisa import _lib

    x = torch.zeros((1, 2, 64, 128), dtype=torch.bfloat16)
    good = _lib.view(x)
    bad = _lib.view(x)
    bad.stride_t = 3  # not a multiple of 16 bytes
    rc = _lib.LIB.b2_full_attention(ctypes.byref(good), ctypes.byref(bad), ctypes.byref(good), ctypes.byref(good),
                                    0.1, None, None)
    assert rc == _lib.B2_ERR_INVALID and b"strides" in _lib.LIB.b2_last_error()
    odd = _lib.view(x[..., :120].contiguous())
    rc = _lib.LIB.b2_pisa_forward(ctypes.byref(odd), ctypes.byref(odd), ctypes.byref(odd), ctypes.byref(odd), 1,
                                  0.1, -2, 0, 1, None, None)
    assert rc == _lib.B2_ERR_UNSUPPORTED


def test_size_limits_and_host_call_arguments_are_checked_without_a_gpu():
    from b200_pisa import _lib

    lib = _lib.LIB
    fake = ctypes.c_void_p(16)  # never dereferenced: the checks fail first
    # pairing keeps its overlap triangle in shared memory: at most 608 blocks
    assert lib.b2_pisa_pair(fake, 1, 609, fake, None) == _lib.B2_ERR_UNSUPPORTED
    assert b"608" in lib.b2_last_error()
    assert lib.b2_pisa_pair(None, 1, 144, fake, None) == _lib.B2_ERR_INVALID
    # routing: at most 1024 blocks, sink in {-2, -1, 0}
    assert lib.b2_pisa_route(fake, _lib.B2_BF16, fake, _lib.B2_BF16, None, 1, 1025, 128, 4, 0.1, -2, fake, fake,
                             None) == _lib.B2_ERR_UNSUPPORTED
    assert lib.b2_pisa_route(fake, _lib.B2_BF16, fake, _lib.B2_BF16, None, 1, 144, 128, 4, 0.1, 5, fake, fake,
                             None) == _lib.B2_ERR_INVALID
    # host-memory call: buffers, sizes and the stage split are validated
    host = lib.b2_pisa_forward_spatial_host
    assert host(None, fake, fake, fake, fake, fake, fake, fake, 2, 16, 96, 96, 128, _lib.B2_BF16, 23, 0.088, -2, 4,
                fake, None) == _lib.B2_ERR_INVALID
    assert host(fake, fake, fake, fake, fake, fake, fake, fake, 2, 16, 96, 96, 64, _lib.B2_BF16, 23, 0.088, -2, 4,
                fake, None) == _lib.B2_ERR_INVALID
    assert host(fake, fake, fake, fake, fake, fake, fake, fake, 2, 16, 96, 96, 128, _lib.B2_F32, 23, 0.088, -2, 4,
                fake, None) == _lib.B2_ERR_UNSUPPORTED
    assert host(fake, fake, fake, fake, fake, fake, fake, fake, 2, 16, 96, 96, 128, _lib.B2_BF16, 23, 0.088, -2, 3,
                fake, None) == _lib.B2_ERR_INVALID
    assert b"heads_per_stage" in lib.b2_last_error()


def test_noalloc_statistics_share_the_view_checks():
    """The allocation-free statistics entry runs the same view checks as the
    workspace entry (token order, tiled grid, token count) before any launch."""
    import torch
    from b200_pisa import _lib

    lib = _lib.LIB
    lib.b2_pisa_block_stats_noalloc.restype = ctypes.c_int
    lib.b2_pisa_block_stats_noalloc.argtypes = [ctypes.POINTER(_lib.View)] * 3 + [ctypes.c_int32] + [ctypes.c_void_p] * 7
    fake = ctypes.c_void_p(256)  # never dereferenced: the checks fail first
    x = torch.zeros((1, 2, 1024, 128), dtype=torch.bfloat16)

    def call(v, entry):
        if entry == "noalloc":
            return lib.b2_pisa_block_stats_noalloc(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), _lib.STATS_HYD,
                                                   fake, fake, fake, fake, None, None, None)
        return lib.b2_pisa_block_stats(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), _lib.STATS_HYD,
                                       fake, fake, fake, fake, None, None, fake, None)

    bad_cases = {
        "unknown token order": _lib.view(x, order=7),
        "grid_h <= 0": _lib.view(x, order=_lib.ORDER_TILED8, grid=(0, 32)),
        "grid not divisible by 8": _lib.view(x, order=_lib.ORDER_TILED8, grid=(12, 32)),
        "tokens not a multiple of the frame": _lib.view(x, order=_lib.ORDER_TILED8, grid=(16, 48)),
    }
    for what, v in bad_cases.items():
        for entry in ("noalloc", "workspace"):
            assert call(v, entry) == _lib.B2_ERR_INVALID, (what, entry)
            msg = lib.b2_last_error()
            assert msg, (what, entry)
    lib.b2_noalloc_last_error.restype = ctypes.c_char_p
    assert lib.b2_noalloc_last_error() == lib.b2_last_error()
    # an unknown statistics mode and a missing output are rejected too
    good = _lib.view(x)
    assert lib.b2_pisa_block_stats_noalloc(ctypes.byref(good), ctypes.byref(good), ctypes.byref(good), 9, fake, fake,
                                           fake, fake, None, None, None) == _lib.B2_ERR_INVALID
    assert lib.b2_pisa_block_stats_noalloc(ctypes.byref(good), ctypes.byref(good), ctypes.byref(good),
                                           _lib.STATS_HYD, None, fake, fake, fake, None, None,
                                           None) == _lib.B2_ERR_INVALID


def test_sharded_and_mask_entry_points_check_arguments_without_a_gpu():
    """Host-side checks of the newer entry points fail before any launch:
    output views outside the output buffer, bad mirror / multicast pointers,
    mask arguments; and the workspace layout offsets are ordered and fit."""
    import torch
    from b200_pisa import _lib

    lib = _lib.LIB
    x = torch.zeros((1, 2, 64, 128), dtype=torch.bfloat16)
    v = _lib.view(x)
    fake = ctypes.c_void_p(4096)
    buf = x.data_ptr()
    nbytes = x.numel() * 2
    peers = (ctypes.c_void_p * 1)(ctypes.c_void_p(1 << 20))
    fwd = lib.b2_pisa_forward_mirrored
    # the view reaches one byte past the buffer
    assert fwd(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), 0, 0.1, -2, 0, 1, buf,
               nbytes - 1, peers, 1, fake, None) == _lib.B2_ERR_INVALID
    assert b"out_buffer" in lib.b2_last_error()
    # the view starts before the buffer
    assert fwd(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), 0, 0.1, -2, 0, 1, buf + 16,
               nbytes, peers, 1, fake, None) == _lib.B2_ERR_INVALID
    # too many mirrors, a misaligned mirror
    assert fwd(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), 0, 0.1, -2, 0, 1, buf, nbytes,
               peers, 8, fake, None) == _lib.B2_ERR_INVALID
    bad_peer = (ctypes.c_void_p * 1)(ctypes.c_void_p((1 << 20) + 8))
    assert fwd(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), 0, 0.1, -2, 0, 1, buf, nbytes,
               bad_peer, 1, fake, None) == _lib.B2_ERR_INVALID
    assert lib.b2_pisa_forward_multicast(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), 0, 0.1,
                                         -2, 0, 1, buf, nbytes, None, fake, None) == _lib.B2_ERR_INVALID
    # masks: unknown dtype, negative stride, misaligned bias
    pack = lib.b2_pack_block_bias
    assert pack(fake, 9, 0, 64, 1, 1, 64, fake, None) == _lib.B2_ERR_INVALID
    assert pack(fake, 0, -1, 64, 1, 1, 64, fake, None) == _lib.B2_ERR_INVALID
    assert pack(fake, 0, 0, 64, 1, 1, 64, ctypes.c_void_p(4100), None) == _lib.B2_ERR_INVALID
    masked = lib.b2_fixed_block_attention_masked
    assert masked(ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), ctypes.byref(v), 0.1, 0, ctypes.c_void_p(4100),
                  0, None) == _lib.B2_ERR_INVALID
    # workspace layout: ascending offsets inside b2_pisa_workspace_bytes
    offs = (ctypes.c_int64 * _lib.WS_FIELDS)()
    assert lib.b2_pisa_workspace_layout(32, 9216, 128, 23, offs, _lib.WS_FIELDS) == 0
    total = lib.b2_pisa_workspace_bytes(32, 9216, 128, 23)
    values = list(offs)
    assert values == sorted(values) and values[0] == 0 and values[-1] < total
    assert all(o % 256 == 0 for o in values)
    assert lib.b2_pisa_workspace_layout(32, 9216, 64, 23, offs, _lib.WS_FIELDS) == _lib.B2_ERR_INVALID
