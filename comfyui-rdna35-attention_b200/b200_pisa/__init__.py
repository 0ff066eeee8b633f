"""B200 (sm_100a) PISA HYD attention: the drop-in counterpart of the
reference's native wheel ``rdna35_pisa_ck`` (native/rdna35_pisa_ck/
rdna35_pisa_ck/__init__.py).

Same public surface: ``forward``, ``forward_spatial_bhtd``,
``block_stats_hyd``, ``prepare``, ``build_info``, ``capabilities``,
``clear_compile_cache``, the constants, a ``_C`` namespace with the native
entry points (block_stats, block_stats_hyd, pack_spatial_qkv,
unpack_spatial_output, fuse_spatial_epilogue), and ``torch.library`` custom
ops with fake implementations so an outer ``torch.compile(fullgraph=True)``
traces through.  Differences by design: the whole HYD forward (statistics,
routing, exact block-sparse attention, centroid tail, first-order correction
and the merge) runs as CUDA kernels of ``libb200attn.so`` launched through
one C-ABI call, and the spatial path reads the raster [B,T,H,D] layout in
place instead of packing it.
"""
from __future__ import annotations

import ctypes
import functools
import math
import struct
import types

import torch

from . import _lib
from ._lib import LIB, check, ptr, stream_of, view

__version__ = "0.1.0"

BLOCK_SIZE = 64
HEAD_DIM = 128
MAX_BLOCKS = 144
MAX_TOKENS = BLOCK_SIZE * MAX_BLOCKS
SPATIAL_TOKENS = 9216
SPATIAL_SIDE = 96
SPATIAL_SPARSE_EXACT_BLOCKS = 23
GENERIC_MAX_BLOCKS = 1024
_SUPPORTED_DTYPES = {torch.bfloat16}
_NATIVE_API = LIB.b2_api_version()


def _parse_build_info() -> dict[str, object]:
    info: dict[str, object] = {}
    for item in _lib.build_info_string().split(";"):
        key, _, value = item.partition("=")
        info[key] = int(value) if value.lstrip("-").isdigit() else value
    return info


_BUILD_INFO = _parse_build_info()


@functools.lru_cache(maxsize=16)
def _checked_device(index: int) -> int:
    check(LIB.b2_check_device(index))
    return index


def _float32(value: float) -> float:
    try:
        converted = struct.unpack("f", struct.pack("f", float(value)))[0]
    except (OverflowError, struct.error, TypeError, ValueError) as exc:
        raise ValueError("scale must be representable as a positive finite float32 value.") from exc
    if not math.isfinite(converted) or converted <= 0.0:
        raise ValueError("scale must be representable as a positive finite float32 value.")
    return converted


def _on_cuda_device(*tensors: torch.Tensor) -> bool:
    first = tensors[0].device
    return first.type == "cuda" and all(t.device == first for t in tensors)


def _validate_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    # mirrors rdna35_pisa_ck/__init__.py:80-95
    if not all(isinstance(tensor, torch.Tensor) for tensor in (q, k, v)):
        raise TypeError("q, k, and v must be torch tensors.")
    if q.ndim != 3 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("PISA B200 expects matching [BH,T,D] q/k/v tensors.")
    if q.shape[0] <= 0 or q.shape[1] <= 0 or q.shape[1] > MAX_TOKENS or q.shape[2] != HEAD_DIM:
        raise ValueError(f"PISA B200 requires BH>0, 0<T<={MAX_TOKENS}, and D={HEAD_DIM}.")
    if not _on_cuda_device(q, k, v):
        raise ValueError("PISA B200 requires q/k/v on one CUDA device.")
    if q.dtype not in _SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("PISA B200 requires matching bfloat16 q/k/v.")
    if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
        raise ValueError("PISA B200 requires contiguous q/k/v.")
    if q.requires_grad or k.requires_grad or v.requires_grad:
        raise ValueError("PISA B200 is forward-only.")


def _validate_spatial_bhtd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    # mirrors rdna35_pisa_ck/__init__.py:98-123
    if not all(isinstance(tensor, torch.Tensor) for tensor in (q, k, v)):
        raise TypeError("q, k, and v must be torch tensors.")
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("PISA spatial B200 expects matching [B,H,T,D] q/k/v tensors.")
    batch, heads, tokens, head_dim = q.shape
    if batch <= 0 or heads <= 0 or tokens != SPATIAL_TOKENS or head_dim != HEAD_DIM:
        raise ValueError(f"PISA spatial B200 requires B>0, H>0, T={SPATIAL_TOKENS}, and D={HEAD_DIM}.")
    if not _on_cuda_device(q, k, v):
        raise ValueError("PISA spatial B200 requires q/k/v on one CUDA device.")
    if q.dtype not in _SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("PISA spatial B200 requires matching bfloat16 q/k/v.")
    expected_stride = (tokens * heads * head_dim, head_dim, heads * head_dim, 1)
    if q.stride() != expected_stride or k.stride() != expected_stride or v.stride() != expected_stride:
        raise ValueError("PISA spatial B200 requires BHTD views of contiguous [B,T,H,D] storage.")
    if any(tensor.requires_grad for tensor in (q, k, v)):
        raise ValueError("PISA spatial B200 is forward-only.")


def _check_exact_and_sink(exact_blocks, blocks: int, sink_block) -> None:
    if isinstance(exact_blocks, bool) or not isinstance(exact_blocks, int):
        raise TypeError("exact_blocks must be an integer.")
    if exact_blocks < 0 or exact_blocks > blocks:
        raise ValueError(f"exact_blocks must be in [0,{blocks}].")
    if sink_block not in (None, -1, 0):
        raise ValueError("sink_block must be None, -1, or 0.")
    if sink_block is not None and exact_blocks == 0:
        raise ValueError("sink_block requires at least one exact block.")


def _workspace(device: torch.device, batch_heads: int, tokens: int, exact_blocks: int) -> torch.Tensor:
    nbytes = int(LIB.b2_pisa_workspace_bytes(batch_heads, tokens, HEAD_DIM, exact_blocks))
    if nbytes < 0:
        raise ValueError("invalid PISA workspace request")
    return torch.empty(nbytes, device=device, dtype=torch.uint8)


def _native_forward(q_view, k_view, v_view, out_view, ref: torch.Tensor, batch_heads: int, tokens: int,
                    exact_blocks: int, scale: float, sink_block: int, stats_mode: int,
                    first_order: bool) -> torch.Tensor | None:
    """One b2_pisa_forward call; returns the workspace it used (None when dense)."""
    _checked_device(ref.device.index if ref.device.index is not None else torch.cuda.current_device())
    blocks = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    workspace = _workspace(ref.device, batch_heads, tokens, exact_blocks) if exact_blocks < blocks else None
    check(
        LIB.b2_pisa_forward(
            ctypes_ref(q_view), ctypes_ref(k_view), ctypes_ref(v_view), ctypes_ref(out_view), exact_blocks, scale,
            sink_block, stats_mode, 1 if first_order else 0, ptr(workspace), stream_of(ref),
        )
    )
    return workspace


def _routing_from_workspace(workspace: torch.Tensor, batch_heads: int, tokens: int, exact_blocks: int):
    """(indices int32 [BH,nb,k], h_norm FP32 [BH,nb]) read from a sparse
    b2_pisa_forward workspace at the offsets b2_pisa_workspace_layout reports."""
    blocks = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    offsets = (ctypes.c_int64 * _lib.WS_FIELDS)()
    check(LIB.b2_pisa_workspace_layout(batch_heads, tokens, HEAD_DIM, exact_blocks, offsets, _lib.WS_FIELDS))

    def field(index: int, count: int, dtype: torch.dtype) -> torch.Tensor:
        start = offsets[index]
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return workspace[start:start + nbytes].view(dtype)

    indices = field(_lib.WS_INDICES, batch_heads * blocks * exact_blocks, torch.int32)
    h_norm = field(_lib.WS_HNORM, batch_heads * blocks, torch.float32)
    return indices.view(batch_heads, blocks, exact_blocks).clone(), h_norm.view(batch_heads, blocks).clone()


def forward_spatial_bhtd_with_routing(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                                      scale: float | None = None, sink_block: int | None = None):
    """Diagnostics form of forward_spatial_bhtd: (output, indices, h_norm),
    where indices int32 [B*H,144,exact_blocks] are the key blocks the call
    routed each query block to (ascending, block-major order) and h_norm FP32
    [B*H,144] the covariance norms behind the routing bias.  Same kernels and
    output as forward_spatial_bhtd; sparse calls only."""
    _validate_spatial_bhtd(q, k, v)
    blocks = SPATIAL_TOKENS // BLOCK_SIZE
    _check_exact_and_sink(exact_blocks, blocks, sink_block)
    if not 0 < exact_blocks < blocks:
        raise ValueError("routing is only produced by sparse calls (0 < exact_blocks < 144).")
    scale_value = _float32(1.0 / math.sqrt(HEAD_DIM) if scale is None else scale)
    batch, heads, tokens, head_dim = q.shape
    out = torch.empty((batch, tokens, heads * head_dim), device=q.device, dtype=q.dtype)
    qv, kv, vv, ov = _spatial_views(q, k, v, out)
    ws = _native_forward(qv, kv, vv, ov, q, batch * heads, tokens, exact_blocks, scale_value,
                         -2 if sink_block is None else sink_block, _lib.STATS_HYD, True)
    indices, h_norm = _routing_from_workspace(ws, batch * heads, tokens, exact_blocks)
    return out, indices, h_norm


def ctypes_ref(v):
    import ctypes

    return ctypes.byref(v)


# ---------------------------------------------------------------- custom ops
@torch.library.custom_op("b200_pisa::block_stats_hyd", mutates_args=(), device_types="cuda")
def _block_stats_hyd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return _C.block_stats_hyd(q, k, v)


@_block_stats_hyd_op.register_fake
def _block_stats_hyd_op_fake(q, k, v):
    del k, v
    blocks = (q.shape[1] + BLOCK_SIZE - 1) // BLOCK_SIZE
    shape = (q.shape[0], blocks, q.shape[2])
    return (
        q.new_empty(shape),
        q.new_empty(shape, dtype=torch.float32),
        q.new_empty(shape),
        q.new_empty((q.shape[0], q.shape[2], q.shape[2]), dtype=torch.float32),
        q.new_empty((q.shape[0], blocks), dtype=torch.float32),
    )


@torch.library.custom_op("b200_pisa::forward", mutates_args=(), device_types="cuda")
def _forward_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int, scale: float, sink_block: int) -> torch.Tensor:
    out = torch.empty_like(q)
    _native_forward(view(q), view(k), view(v), view(out), q, q.shape[0], q.shape[1], exact_blocks, scale, sink_block,
                    _lib.STATS_HYD, True)
    return out


@_forward_op.register_fake
def _forward_op_fake(q, k, v, exact_blocks, scale, sink_block):
    del k, v, exact_blocks, scale, sink_block
    return torch.empty_like(q)


def _spatial_views(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor):
    grid = (SPATIAL_SIDE, SPATIAL_SIDE)
    batch, heads, tokens, head_dim = q.shape
    out_bhtd = out.view(batch, tokens, heads, head_dim).permute(0, 2, 1, 3)
    tiled = dict(order=_lib.ORDER_TILED8, grid=grid)
    return view(q, **tiled), view(k, **tiled), view(v, **tiled), view(out_bhtd, **tiled)


@torch.library.custom_op("b200_pisa::forward_spatial_bhtd", mutates_args=(), device_types="cuda")
def _forward_spatial_bhtd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int, scale: float, sink_block: int) -> torch.Tensor:
    batch, heads, tokens, head_dim = q.shape
    out = torch.empty((batch, tokens, heads * head_dim), device=q.device, dtype=q.dtype)
    qv, kv, vv, ov = _spatial_views(q, k, v, out)
    _native_forward(qv, kv, vv, ov, q, batch * heads, tokens, exact_blocks, scale, sink_block, _lib.STATS_HYD, True)
    return out


@_forward_spatial_bhtd_op.register_fake
def _forward_spatial_bhtd_op_fake(q, k, v, exact_blocks, scale, sink_block):
    del k, v, exact_blocks, scale, sink_block
    return q.new_empty((q.shape[0], q.shape[2], q.shape[1] * q.shape[3]))


# ---------------------------------------------------------------- public API
def block_stats_hyd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """(q_centroids BF16, k_centroids FP32, v_means BF16, h_sum FP32); mirrors
    rdna35_pisa_ck/__init__.py:215-230."""
    if q.ndim != 3 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("PISA B200 HYD expects matching [BH,T,D] q/k/v tensors.")
    if q.shape[0] <= 0 or q.shape[1] <= 0 or q.shape[1] > MAX_TOKENS or q.shape[2] != HEAD_DIM:
        raise ValueError(f"PISA B200 HYD requires BH>0, 0<T<={MAX_TOKENS}, and D={HEAD_DIM}.")
    if not _on_cuda_device(q, k, v):
        raise ValueError("PISA B200 HYD requires q/k/v on one CUDA device.")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("PISA B200 HYD requires matching fp16/bf16 q/k/v.")
    if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
        raise ValueError("PISA B200 HYD requires contiguous q/k/v.")
    if q.requires_grad or k.requires_grad or v.requires_grad:
        raise ValueError("PISA B200 HYD is forward-only.")
    return _block_stats_hyd_op(q, k, v)[:4]


def forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int, scale: float | None = None,
            sink_block: int | None = None) -> torch.Tensor:
    """PISA HYD forward on contiguous [BH,T,128] BF16 (rdna35_pisa_ck/__init__.py:381-403)."""
    _validate_qkv(q, k, v)
    blocks = (q.shape[1] + BLOCK_SIZE - 1) // BLOCK_SIZE
    _check_exact_and_sink(exact_blocks, blocks, sink_block)
    scale_value = _float32(1.0 / math.sqrt(HEAD_DIM) if scale is None else scale)
    return _forward_op(q, k, v, exact_blocks, scale_value, -2 if sink_block is None else sink_block)


def forward_spatial_bhtd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                         scale: float | None = None, sink_block: int | None = None) -> torch.Tensor:
    """Anima spatial PISA: BHTD views of [B,9216,H,128] BF16 -> [B,9216,H*128]
    raster output (rdna35_pisa_ck/__init__.py:406-433)."""
    _validate_spatial_bhtd(q, k, v)
    blocks = SPATIAL_TOKENS // BLOCK_SIZE
    _check_exact_and_sink(exact_blocks, blocks, sink_block)
    if exact_blocks not in (SPATIAL_SPARSE_EXACT_BLOCKS, blocks):
        raise ValueError(
            f"spatial PISA supports exact_blocks={SPATIAL_SPARSE_EXACT_BLOCKS}; "
            f"use exact_blocks={blocks} only for dense SDPA validation."
        )
    scale_value = _float32(1.0 / math.sqrt(HEAD_DIM) if scale is None else scale)
    return _forward_spatial_bhtd_op(q, k, v, exact_blocks, scale_value, -2 if sink_block is None else sink_block)


def forward_spatial_bhtd_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                              scale: float | None = None, sink_block: int | None = None, *,
                              device: torch.device | int | None = None, heads_per_stage: int = 4,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """forward_spatial_bhtd for activations held in host memory: q/k/v are
    BHTD views of page-locked [B,9216,H,128] BF16 raster storage on the CPU;
    returns the [B,9216,H*128] raster output in page-locked host memory (or
    writes ``out``).  The call runs in stages of ``heads_per_stage`` heads of
    one batch so that the PCIe copies of one stage overlap the compute of its
    neighbours (b2_pisa_forward_spatial_host).  Results are identical to
    forward_spatial_bhtd on the same values.  The output is complete once the
    device's current stream has been synchronised."""
    if not all(isinstance(tensor, torch.Tensor) for tensor in (q, k, v)):
        raise TypeError("q, k, and v must be torch tensors.")
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("PISA spatial B200 expects matching [B,H,T,D] q/k/v tensors.")
    batch, heads, tokens, head_dim = q.shape
    if tokens != SPATIAL_TOKENS or head_dim != HEAD_DIM:
        raise ValueError(f"PISA spatial B200 requires B>0, H>0, T={SPATIAL_TOKENS}, and D={HEAD_DIM}.")
    if q.dtype not in _SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("PISA spatial B200 requires matching bfloat16 q/k/v.")
    expected_stride = (tokens * heads * head_dim, head_dim, heads * head_dim, 1)
    if q.stride() != expected_stride or k.stride() != expected_stride or v.stride() != expected_stride:
        raise ValueError("PISA spatial B200 requires BHTD views of contiguous [B,T,H,D] storage.")
    if any(t.is_cuda or not t.is_pinned() for t in (q, k, v)):
        raise ValueError("host PISA requires q/k/v in page-locked (pinned) host memory.")
    if heads_per_stage <= 0 or heads % heads_per_stage:
        raise ValueError("heads_per_stage must divide the number of heads.")
    blocks = SPATIAL_TOKENS // BLOCK_SIZE
    _check_exact_and_sink(exact_blocks, blocks, sink_block)
    if exact_blocks not in (SPATIAL_SPARSE_EXACT_BLOCKS, blocks):
        raise ValueError(
            f"spatial PISA supports exact_blocks={SPATIAL_SPARSE_EXACT_BLOCKS}; "
            f"use exact_blocks={blocks} only for dense SDPA validation."
        )
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        dev = torch.device("cuda", device)
    else:
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
    _checked_device(dev.index)
    if out is None:
        out = torch.empty((batch, tokens, heads * head_dim), dtype=q.dtype).pin_memory()
    elif out.shape != (batch, tokens, heads * head_dim) or not out.is_contiguous() or not out.is_pinned():
        raise ValueError("out must be a contiguous pinned [B,T,H*D] host tensor.")
    raster = (batch, tokens, heads, head_dim)
    q_dev, k_dev, v_dev, o_dev = (torch.empty(raster, dtype=q.dtype, device=dev) for _ in range(4))
    ws = _workspace(dev, heads_per_stage, tokens, exact_blocks) if exact_blocks < blocks else None
    scale_value = _float32(1.0 / math.sqrt(HEAD_DIM) if scale is None else scale)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        check(LIB.b2_pisa_forward_spatial_host(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), q_dev.data_ptr(), k_dev.data_ptr(),
            v_dev.data_ptr(), o_dev.data_ptr(), batch, heads, SPATIAL_SIDE, SPATIAL_SIDE, head_dim, _lib.B2_BF16,
            exact_blocks, scale_value, -2 if sink_block is None else sink_block, heads_per_stage, ptr(ws),
            stream.cuda_stream))
    # the device buffers were allocated on `stream`, which waits for the last
    # copy-out, so the caching allocator reuses them only after the copies
    return out


def generic_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int, scale: float,
                    first_order: bool = True, grid: tuple[int, int] | None = None,
                    out: torch.Tensor | None = None, return_indices: bool = False):
    """Generic PISA (generic_pisa.py:141-232 semantics): FP32 centroids,
    routing without the HYD bias, 16-bit-rounded centred K, optional
    first-order term.  q/k/v: [BH,T,D] or [B,H,T,D] views (fp16/bf16,
    head dimension contiguous, D <= 128 a multiple of 8: the kernels' TMA
    tiles read the columns past D as zeros, so no padded copy is made), T up
    to 65536.  grid=(h, w) reads the tokens
    in 8x8-tile order of per-frame h x w rasters (no packing copy); the
    output (``out`` view or a new tensor shaped like q) is in token order.
    return_indices=True also returns the routed key blocks, int32
    [BH,nb,exact_blocks] ascending (diagnostics; sparse calls only)."""
    if q.ndim not in (3, 4) or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("generic PISA requires matching [BH,T,D] or [B,H,T,D] q/k/v")
    if q.shape[-1] > HEAD_DIM or q.shape[-1] % 8:
        raise ValueError(f"B200 generic PISA requires D <= {HEAD_DIM}, a multiple of 8")
    tokens = q.shape[-2]
    blocks = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    if blocks > GENERIC_MAX_BLOCKS:
        raise ValueError(f"B200 generic PISA supports at most {GENERIC_MAX_BLOCKS * BLOCK_SIZE} tokens")
    if not (0 <= exact_blocks <= blocks):
        raise ValueError(f"exact_blocks must be in [0,{blocks}].")
    if out is None:
        out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    order = dict(order=_lib.ORDER_TILED8, grid=tuple(grid)) if grid is not None else {}
    views = [view(x, **order) for x in (q, k, v, out)]
    bh = q.shape[0] * (q.shape[1] if q.ndim == 4 else 1)
    ws = _native_forward(*views, q, bh, tokens, int(exact_blocks), _float32(scale), -2, _lib.STATS_GENERIC,
                         first_order)
    if return_indices:
        if not 0 < exact_blocks < blocks:
            raise ValueError("routing is only produced by sparse calls.")
        return out, _routing_from_workspace(ws, bh, tokens, int(exact_blocks))[0]
    return out


def full_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None) -> torch.Tensor:
    """Exact softmax(q k^T scale) v over [B,H,T,D] / [BH,T,D] views (no mask)."""
    _checked_device(q.device.index if q.device.index is not None else torch.cuda.current_device())
    if out is None:
        out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    check(LIB.b2_full_attention(ctypes_ref(view(q)), ctypes_ref(view(k)), ctypes_ref(view(v)), ctypes_ref(view(out)),
                                _float32(scale), ptr(lse), stream_of(q)))
    return out


_MASK_CODES = {torch.bool: 0, torch.float32: 1, torch.float16: 2, torch.bfloat16: 3}


def block_mask_bias(mask: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Pack a [N,T,T] mask view (N = B*H, or 1 for a mask shared by every
    (batch, head); any strides) into the FP32 [N,T,64] diagonal-block terms
    the masked fixed-block kernels add to the scores (b2_pack_block_bias).
    Returns (bias, bias_bh_stride): the stride is T*64, or 0 when N == 1."""
    if mask.ndim != 3 or mask.shape[1] != mask.shape[2] or mask.dtype not in _MASK_CODES or not mask.is_cuda:
        raise ValueError("block_mask_bias expects a CUDA [N,T,T] bool or float mask")
    n, tokens, _ = mask.shape
    bias = torch.empty((n, tokens, BLOCK_SIZE), device=mask.device, dtype=torch.float32)
    sb, st, sk = mask.stride()
    check(LIB.b2_pack_block_bias(mask.data_ptr(), _MASK_CODES[mask.dtype], sb, st, sk, n, tokens, bias.data_ptr(),
                                 stream_of(mask)))
    return bias, (tokens * BLOCK_SIZE if n > 1 else 0)


def fixed_block_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool = False,
                          out: torch.Tensor | None = None, mask_bias: torch.Tensor | None = None,
                          mask_bias_stride: int = 0) -> torch.Tensor:
    """64-token block-diagonal attention over [B,H,T,D] / [BH,T,D] views;
    ``mask_bias`` (from block_mask_bias) adds each row's mask terms."""
    _checked_device(q.device.index if q.device.index is not None else torch.cuda.current_device())
    if out is None:
        out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    check(LIB.b2_fixed_block_attention_masked(ctypes_ref(view(q)), ctypes_ref(view(k)), ctypes_ref(view(v)),
                                              ctypes_ref(view(out)), _float32(scale), 1 if causal else 0,
                                              ptr(mask_bias), int(mask_bias_stride), stream_of(q)))
    return out


def pack_views(tensors: list[torch.Tensor]) -> torch.Tensor:
    """Copy 1..3 equal-shape [B,H,T,D] views into one contiguous [n,B,H,T,D]
    allocation (minimax_h3_gfx1151_attention.py:64-74)."""
    import ctypes

    n = len(tensors)
    views = (_lib.View * n)(*[view(t) for t in tensors])
    out = torch.empty((n, *tensors[0].shape), device=tensors[0].device, dtype=tensors[0].dtype)
    check(LIB.b2_h3_pack(views, n, ctypes.c_void_p(out.data_ptr()), stream_of(tensors[0])))
    return out


def _native_block_stats(q, k, v, mode: int):
    bh, tokens, dim = q.shape
    blocks = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    _checked_device(q.device.index if q.device.index is not None else torch.cuda.current_device())
    cent_dtype = torch.float32 if mode == _lib.STATS_GENERIC else q.dtype
    q_centroids = torch.empty((bh, blocks, dim), device=q.device, dtype=cent_dtype)
    k_centroids = torch.empty((bh, blocks, dim), device=q.device, dtype=torch.float32)
    v_stats = torch.empty((bh, blocks, dim), device=q.device, dtype=cent_dtype)
    h_sum = torch.empty((bh, dim, dim), device=q.device, dtype=torch.float32)
    h_norm = torch.empty((bh, blocks), device=q.device, dtype=torch.float32)
    workspace = torch.empty(int(LIB.b2_stats_workspace_bytes(bh, tokens, dim)), device=q.device, dtype=torch.uint8)
    check(LIB.b2_pisa_block_stats(ctypes_ref(view(q)), ctypes_ref(view(k)), ctypes_ref(view(v)), mode,
                                  ptr(q_centroids), ptr(k_centroids), ptr(v_stats), ptr(h_sum), ptr(h_norm), None,
                                  ptr(workspace), stream_of(q)))
    return q_centroids, k_centroids, v_stats, h_sum, h_norm


def generic_block_stats(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """(q_centroids FP32, k_centroids FP32, v_sums FP32, h_sum FP32) with the
    semantics of generic_pisa.py:106-138 / pisa_kernel.py:49-84."""
    return _native_block_stats(q, k, v, _lib.STATS_GENERIC)[:4]


def _spatial_grid_view(x: torch.Tensor, batch: int, heads: int):
    return view(x, order=_lib.ORDER_TILED8, grid=(SPATIAL_SIDE, SPATIAL_SIDE))


def _pack_spatial_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Raster BHTD views -> three contiguous block-major [B*H,9216,128]
    tensors (pisa_kernels.cu:638-676)."""
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("PISA spatial QKV pack expects matching [B,H,T,D] q/k/v.")
    batch, heads, tokens, dim = q.shape
    if tokens != SPATIAL_TOKENS or dim != HEAD_DIM:
        raise ValueError("PISA spatial QKV pack requires B>0, H>0, T=9216, and D=128.")
    expected = (tokens * heads * dim, dim, heads * dim, 1)
    for name, x in (("q", q), ("k", k), ("v", v)):
        if x.stride() != expected:
            raise ValueError(f"{name} must be a [B,H,9216,128] view over contiguous [B,9216,H,128] storage.")
    outs = []
    for x in (q, k, v):
        packed = torch.empty((batch * heads, tokens, dim), device=x.device, dtype=x.dtype)
        check(LIB.b2_pack_rows(ctypes_ref(_spatial_grid_view(x, batch, heads)), ptr(packed), stream_of(x)))
        outs.append(packed)
    return tuple(outs)


def _unpack_spatial_output(output: torch.Tensor, batch: int, heads: int) -> torch.Tensor:
    """Block-major [B*H,9216,128] -> raster [B,9216,H*128] (pisa_kernels.cu:679-707)."""
    if output.ndim != 3 or output.shape != (batch * heads, SPATIAL_TOKENS, HEAD_DIM) or not output.is_contiguous():
        raise ValueError("PISA spatial output unpack expects contiguous [B*H,9216,128] input.")
    unpacked = torch.empty((batch, SPATIAL_TOKENS, heads * HEAD_DIM), device=output.device, dtype=output.dtype)
    dst = unpacked.view(batch, SPATIAL_TOKENS, heads, HEAD_DIM).permute(0, 2, 1, 3)
    check(LIB.b2_unpack_rows(ptr(output), ctypes_ref(_spatial_grid_view(dst, batch, heads)), stream_of(output)))
    return unpacked


def _fuse_spatial_epilogue(exact_output, exact_lse, approximate_output, approximate_lse, correction, batch: int,
                           heads: int) -> torch.Tensor:
    """LSE-weighted merge + raster scatter (pisa_kernels.cu:710-773)."""
    bh = batch * heads
    for name, x in (("exact output", exact_output), ("approximate output", approximate_output)):
        if x.shape != (bh, SPATIAL_TOKENS, HEAD_DIM) or not x.is_contiguous() or x.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be contiguous bfloat16 [B*H,9216,128].")
    if correction.shape != (bh, SPATIAL_TOKENS, HEAD_DIM) or correction.dtype != torch.float32 or not correction.is_contiguous():
        raise ValueError("correction must be contiguous float32 [B*H,9216,128].")
    for name, x in (("exact LSE", exact_lse), ("approximate LSE", approximate_lse)):
        if x.shape != (bh, SPATIAL_TOKENS) or x.dtype != torch.float32 or not x.is_contiguous():
            raise ValueError(f"{name} must be contiguous float32 [B*H,9216].")
    out = torch.empty((batch, SPATIAL_TOKENS, heads * HEAD_DIM), device=exact_output.device, dtype=exact_output.dtype)
    dst = out.view(batch, SPATIAL_TOKENS, heads, HEAD_DIM).permute(0, 2, 1, 3)
    check(LIB.b2_merge_epilogue(ptr(exact_output), ptr(exact_lse), ptr(approximate_output), ptr(approximate_lse),
                                ptr(correction), ctypes_ref(_spatial_grid_view(dst, batch, heads)),
                                stream_of(exact_output)))
    return out


def _c_block_stats(q, k, v):
    out = _native_block_stats(q, k, v, _lib.STATS_SCALED)
    return out[0], out[1], out[2]


_C = types.SimpleNamespace(
    block_stats=_c_block_stats,
    block_stats_hyd=lambda q, k, v: _native_block_stats(q, k, v, _lib.STATS_HYD),
    pack_spatial_qkv=_pack_spatial_qkv,
    unpack_spatial_output=_unpack_spatial_output,
    fuse_spatial_epilogue=_fuse_spatial_epilogue,
    build_info=lambda: dict(_BUILD_INFO),
)


def prepare(device_index: int | None = None) -> None:
    """Validate the device once (the reference pre-builds Flex block masks)."""
    if not torch.cuda.is_available():
        raise RuntimeError("b200_pisa requires a CUDA device.")
    index = torch.cuda.current_device() if device_index is None else int(device_index)
    _checked_device(index)


def build_info() -> dict[str, object]:
    return {
        **_BUILD_INFO,
        "package_version": __version__,
        "torch_runtime_version": torch.__version__,
        "cuda_runtime_version": torch.version.cuda,
    }


def capabilities() -> dict[str, object]:
    return {
        "architecture": "sm_100a",
        "block_size": BLOCK_SIZE,
        "head_dim": HEAD_DIM,
        "max_blocks": MAX_BLOCKS,
        "dtypes": (torch.bfloat16,),
        "causal": False,
        "backward": False,
        "first_order_tail": True,
        "first_order_routing_bias": True,
        "flex_attention": False,
        "fused_tail": True,
        "outer_torch_compile": True,
        "outer_torch_compile_requires_prepare": False,
        "spatial_bhtd": True,
        "spatial_tokens": SPATIAL_TOKENS,
        "spatial_sparse_exact_blocks": (SPATIAL_SPARSE_EXACT_BLOCKS,),
        "hyd_stats_head_dims": (128,),
        "hyd_stats_dtypes": (torch.bfloat16,),
        "generic_max_tokens": GENERIC_MAX_BLOCKS * BLOCK_SIZE,
    }


def clear_compile_cache() -> None:
    _checked_device.cache_clear()


__all__ = [
    "BLOCK_SIZE",
    "HEAD_DIM",
    "MAX_BLOCKS",
    "SPATIAL_SPARSE_EXACT_BLOCKS",
    "SPATIAL_TOKENS",
    "block_mask_bias",
    "block_stats_hyd",
    "build_info",
    "capabilities",
    "clear_compile_cache",
    "fixed_block_attention",
    "forward",
    "forward_spatial_bhtd",
    "forward_spatial_bhtd_with_routing",
    "full_attention",
    "generic_block_stats",
    "generic_forward",
    "pack_views",
    "prepare",
]
