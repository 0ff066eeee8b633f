"""ctypes binding of the in-tree C-ABI library ``lib/libb200attn.so``.

The library is the only compute path: importing this module fails loudly when
the shared object is missing (build it with ``build_native.py``), and every
call raises ``RuntimeError`` with the library's message when an entry point
returns a non-zero status.  Tensors cross the boundary as ``b2_view`` structs
(base pointer, element strides, shape, dtype, token order) built from torch
tensors; launches go on the tensor device's current CUDA stream.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

import torch

LIB_PATH = pathlib.Path(os.environ.get("B200ATTN_LIB", pathlib.Path(__file__).resolve().parent / "lib" / "libb200attn.so"))

B2_OK = 0
B2_ERR_INVALID = 1
B2_ERR_UNSUPPORTED = 2
B2_ERR_CUDA = 3
B2_ERR_DEVICE = 4

B2_BF16, B2_F16, B2_F32 = 0, 1, 2
ORDER_LINEAR, ORDER_TILED8 = 0, 1
STATS_HYD, STATS_GENERIC, STATS_SCALED = 0, 1, 2
# workspace buffer indices of b2_pisa_workspace_layout (B2_WS_* in the header)
WS_QC, WS_KC, WS_HSUM, WS_HNORM, WS_INDICES, WS_SEL, WS_FIELDS = 0, 1, 3, 5, 8, 9, 12

_DTYPE_CODES = {torch.bfloat16: B2_BF16, torch.float16: B2_F16, torch.float32: B2_F32}

# Every symbol include/b200attn.h declares, with (restype, argtypes).
_VP = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float


class View(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("stride_t", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("order", ctypes.c_int32),
        ("grid_h", ctypes.c_int32),
        ("grid_w", ctypes.c_int32),
    ]


_VIEW_P = ctypes.POINTER(View)

SIGNATURES: dict[str, tuple] = {
    "b2_last_error": (ctypes.c_char_p, []),
    "b2_last_kernel": (ctypes.c_char_p, []),
    "b2_read_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32)]),
    "b2_set_trace": (ctypes.c_int, [ctypes.c_void_p]),
    "b2_debug_withhold_q": (ctypes.c_int, [_I32]),
    "b2_api_version": (ctypes.c_int, []),
    "b2_build_info": (ctypes.c_int, [ctypes.c_char_p, _I64]),
    "b2_check_device": (ctypes.c_int, [ctypes.c_int]),
    "b2_stats_workspace_bytes": (_I64, [_I32, _I32, _I32]),
    "b2_pisa_block_stats": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "b2_pisa_route": (ctypes.c_int, [_VP, _I32, _VP, _I32, _VP, _I32, _I32, _I32, _I32, _F32, _I32, _VP, _VP, _VP]),
    "b2_pisa_attention": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _VP, _I32, _VP, _VP, _VP, _VP, _VP, _F32, _VP, _VP]),
    "b2_pisa_pair": (ctypes.c_int, [_VP, _I32, _I32, _VP, _VP]),
    "b2_pisa_workspace_bytes": (_I64, [_I32, _I32, _I32, _I32]),
    "b2_pisa_workspace_layout": (ctypes.c_int, [_I32, _I32, _I32, _I32, ctypes.POINTER(_I64), _I32]),
    "b2_pisa_forward": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _I32, _F32, _I32, _I32, _I32, _VP, _VP]),
    "b2_pisa_forward_mirrored": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _I32, _F32, _I32, _I32, _I32, _VP,
                                                _I64, ctypes.POINTER(_VP), _I32, _VP, _VP]),
    "b2_pisa_forward_multicast": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _I32, _F32, _I32, _I32, _I32, _VP,
                                                 _I64, _VP, _VP, _VP]),
    "b2_pisa_forward_spatial_host": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I32, _I32, _I32, _I32,
                                                    _I32, _I32, _I32, _F32, _I32, _I32, _VP, _VP]),
    "b2_full_attention": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _F32, _VP, _VP]),
    "b2_fixed_block_attention": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _F32, _I32, _VP]),
    "b2_fixed_block_attention_masked": (ctypes.c_int, [_VIEW_P, _VIEW_P, _VIEW_P, _VIEW_P, _F32, _I32, _VP, _I64,
                                                       _VP]),
    "b2_pack_block_bias": (ctypes.c_int, [_VP, _I32, _I64, _I64, _I64, _I32, _I32, _VP, _VP]),
    "b2_pack_rows": (ctypes.c_int, [_VIEW_P, _VP, _VP]),
    "b2_unpack_rows": (ctypes.c_int, [_VP, _VIEW_P, _VP]),
    "b2_merge_epilogue": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _VIEW_P, _VP]),
    "b2_h3_pack": (ctypes.c_int, [_VIEW_P, _I32, _VP, _VP]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"B200 attention library not found at {LIB_PATH}; build it with "
            "`python comfyui-rdna35-attention_b200/build_native.py` (nvcc 12.9, sm_100a)."
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


LIB = _load()


class NativeError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(code: int) -> None:
    if code != B2_OK:
        message = LIB.b2_last_error().decode(errors="replace")
        if code in (B2_ERR_INVALID, B2_ERR_UNSUPPORTED):
            raise ValueError(message)
        raise NativeError(code, message)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {dtype}") from exc


def view(tensor: torch.Tensor, *, order: int = ORDER_LINEAR, grid: tuple[int, int] = (0, 0)) -> View:
    """b2_view of a [B,H,T,D] (or [BH,T,D], read as B=BH, H=1) tensor."""
    if tensor.ndim == 3:
        bh, tokens, dim = tensor.shape
        sb, st, sd = tensor.stride()
        batch, heads, sh = bh, 1, 0
    elif tensor.ndim == 4:
        batch, heads, tokens, dim = tensor.shape
        sb, sh, st, sd = tensor.stride()
    else:
        raise ValueError(f"expected a rank-3 or rank-4 tensor, got rank {tensor.ndim}")
    if sd != 1 and dim > 1:
        raise ValueError("the head dimension must be contiguous (stride 1)")
    return View(
        tensor.data_ptr(), sb, sh, st, batch, heads, tokens, dim, dtype_code(tensor.dtype), order, grid[0], grid[1]
    )


def stream_of(tensor: torch.Tensor) -> int:
    return torch.cuda.current_stream(tensor.device).cuda_stream


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def build_info_string() -> str:
    buffer = ctypes.create_string_buffer(512)
    check(LIB.b2_build_info(buffer, len(buffer)))
    return buffer.value.decode()


def last_kernel() -> str:
    """Attention kernel this thread launched last ("tcgen05" or "mma_sync")."""
    return LIB.b2_last_kernel().decode()


def read_status() -> int:
    """Read and clear the device status word (synchronises the device)."""
    value = ctypes.c_int32(0)
    check(LIB.b2_read_status(ctypes.byref(value)))
    return value.value


class PipelineTimeout(RuntimeError):
    """A kernel's bounded pipeline wait ran out; its outputs are invalid."""

    def __init__(self, status: int):
        super().__init__(f"B200 attention pipeline wait timed out at site {status & 0xFF} "
                         f"(status word 0x{status:x}); the launch's outputs are invalid")
        self.status = status
        self.site = status & 0xFF


def check_status() -> None:
    """Read and clear the device status word; raise PipelineTimeout when a
    kernel since the last read gave up on a pipeline wait."""
    status = read_status()
    if status != 0:
        raise PipelineTimeout(status)
