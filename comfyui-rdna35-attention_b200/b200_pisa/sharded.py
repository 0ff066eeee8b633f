"""Head-sharded PISA across the GPUs of one node.

Every (batch, head) of a PISA call is independent: the statistics, routing
and attention of one head never read another head's data (the reference's
kernels grid over batch*heads, native/rdna35_pisa_ck/csrc/pisa_kernels.cu:583,
and its FlexAttention call is per (batch, head)).  A call over H heads on N
GPUs (one process per GPU, torch.distributed) therefore splits the heads
into N contiguous ranges, each rank computing its range with the single-GPU
kernels.  The outputs are exchanged in one of two ways:

* ``exchange="multicast"`` / ``"peer"``: the output lives in a symmetric
  buffer (``torch.distributed._symmetric_memory``: every rank's copy mapped
  into every process) and the attention kernel's epilogue, after its local
  store, writes each output row (staged in shared memory, whole 256-byte
  rows) either once through the buffer's NVLink multicast address, which the
  NVSwitch replicates into every GPU's copy (``b2_pisa_forward_multicast``),
  or into each peer's copy in turn (``b2_pisa_forward_mirrored``); two
  device-side barriers bracket the call.  ``"auto"`` (default) uses the
  peer stores: measured on 8 GPUs, 0.259 ms per call against 0.275 ms with
  multicast (2 GPUs: 0.381 / 0.378 ms).
* ``exchange="nccl"``: each rank computes into a local [B,T,Hs*D] buffer, one
  NCCL all-gather exchanges the shards and a 16-byte copy kernel interleaves
  the gathered [N,B,T,Hs*D] shards into the [B,T,H*D] raster.

Because a head's output does not depend on which other heads share its call,
the sharded result equals the single-GPU result bit for bit.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_SYMMETRIC: dict = {}
_SYMMETRIC_UNAVAILABLE: set = set()  # why the automatic exchange fell back to NCCL


def head_range(heads: int, world: int, rank: int) -> tuple[int, int]:
    """[h0, h1) of the heads rank `rank` of `world` computes: equal
    contiguous ranges (the all-gather exchanges equal-sized shards)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    if heads <= 0 or heads % world:
        raise ValueError(f"{heads} heads cannot be split evenly over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def interleave_shards(gathered: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[N,B,T,W] rank-major shards -> [B,T,N*W] with shard n in columns
    [n*W, (n+1)*W).  On CUDA tensors this is the library's 16-byte row-copy
    kernel (b2_unpack_rows over a strided destination view); host tensors
    (the gloo tests of the exchange logic) use a torch permute."""
    world, batch, tokens, width = gathered.shape
    if out is None:
        out = torch.empty((batch, tokens, world * width), device=gathered.device, dtype=gathered.dtype)
    if out.shape != (batch, tokens, world * width) or not out.is_contiguous() or out.dtype != gathered.dtype:
        raise ValueError("out must be a contiguous [B,T,N*W] tensor of the shards' dtype")
    if not gathered.is_cuda:
        out.copy_(gathered.permute(1, 2, 0, 3).reshape(batch, tokens, world * width))
        return out
    src = gathered.contiguous()
    # destination rows: "batch" = shard n (column offset n*W), "heads" = b
    dst = _lib.View(out.data_ptr(), width, tokens * world * width, world * width, world, batch, tokens, width,
                    _lib.dtype_code(out.dtype), _lib.ORDER_LINEAR, 0, 0)
    _lib.check(_lib.LIB.b2_unpack_rows(src.data_ptr(), ctypes.byref(dst), _lib.stream_of(out)))
    return out


def gather_head_shards(local: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather each rank's [B,T,Hs*D] output over the process group (one
    NCCL all_gather_into_tensor on GPUs) and return the [B,T,N*Hs*D] raster."""
    world = dist.get_world_size(group)
    local = local.contiguous()
    if world == 1:
        if out is None:
            return local
        out.copy_(local)
        return out
    gathered = torch.empty((world * local.shape[0], *local.shape[1:]), device=local.device, dtype=local.dtype)
    dist.all_gather_into_tensor(gathered, local, group=group)
    return interleave_shards(gathered.view(world, *local.shape), out)


def _symmetric_output(shape: tuple, dtype: torch.dtype, device: torch.device, group):
    """(buffer, handle) of a symmetric [B,T,H*D] output buffer for `group`,
    allocated and exchanged once per (shape, dtype, device, group)."""
    import torch.distributed._symmetric_memory as symm_mem

    group = group if group is not None else dist.group.WORLD
    key = (tuple(shape), dtype, device, group.group_name)
    if key not in _SYMMETRIC:
        buf = symm_mem.empty(shape, dtype=dtype, device=device)
        handle = symm_mem.rendezvous(buf, group)
        _SYMMETRIC[key] = (buf, handle)
    return _SYMMETRIC[key]


def forward_spatial_bhtd_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                                 scale: float | None = None, sink_block: int | None = None, *, group=None,
                                 out: torch.Tensor | None = None, exchange: str = "auto") -> torch.Tensor:
    """Anima spatial PISA over the heads of all ranks of `group`.

    q/k/v: this rank's head shard, BHTD views [B,Hs,9216,128] of contiguous
    [B,9216,Hs,128] BF16 storage (heads head_range(H, N, rank) of the full
    call).  Returns the full [B,9216,N*Hs*128] raster output on every rank,
    equal to forward_spatial_bhtd over all H heads on one GPU.  With
    a symmetric-buffer exchange the returned tensor is the group's symmetric output
    buffer, valid until the next peer-exchange call of the same shape on the
    group (pass ``out`` to receive a copy instead)."""
    from . import (HEAD_DIM, SPATIAL_SIDE, _check_exact_and_sink, _checked_device, _float32,
                   _validate_spatial_bhtd, _workspace, forward_spatial_bhtd)

    if exchange not in ("auto", "multicast", "peer", "nccl"):
        raise ValueError("exchange must be 'auto', 'multicast', 'peer' or 'nccl'")
    world = dist.get_world_size(group)
    if exchange == "nccl" or world == 1:
        local = forward_spatial_bhtd(q, k, v, exact_blocks, scale=scale, sink_block=sink_block)
        return gather_head_shards(local, group=group, out=out)
    _validate_spatial_bhtd(q, k, v)
    batch, heads, tokens, dim = q.shape
    blocks = tokens // 64
    _check_exact_and_sink(exact_blocks, blocks, sink_block)
    rank = dist.get_rank(group)
    _checked_device(q.device.index)
    if world - 1 > 7:
        raise ValueError("the peer exchange supports at most 8 ranks")
    try:
        full, handle = _symmetric_output((batch, tokens, world * heads * dim), q.dtype, q.device, group)
    except (RuntimeError, OSError) as exc:
        if exchange != "auto":
            raise
        # no symmetric memory on this system (e.g. no peer access): NCCL exchange
        _SYMMETRIC_UNAVAILABLE.add(str(exc)[:200])
        local = forward_spatial_bhtd(q, k, v, exact_blocks, scale=scale, sink_block=sink_block)
        return gather_head_shards(local, group=group, out=out)
    h0 = rank * heads
    local = full.view(batch, tokens, world * heads, dim)[:, :, h0:h0 + heads]
    tiled = dict(order=_lib.ORDER_TILED8, grid=(SPATIAL_SIDE, SPATIAL_SIDE))
    qv, kv, vv = (_lib.view(x, **tiled) for x in (q, k, v))
    ov = _lib.view(local.permute(0, 2, 1, 3), **tiled)
    peers = [handle.buffer_ptrs[p] for p in range(world) if p != rank]
    mirrors = (ctypes.c_void_p * len(peers))(*peers)
    ws = _workspace(q.device, batch * heads, tokens, exact_blocks) if exact_blocks < blocks else None
    scale_value = _float32(1.0 / (HEAD_DIM ** 0.5) if scale is None else scale)
    multicast = int(getattr(handle, "multicast_ptr", 0) or 0)
    if exchange == "multicast" and not multicast:
        raise ValueError("the symmetric output buffer has no multicast mapping on this system")
    use_multicast = multicast != 0 and exchange == "multicast"
    handle.barrier(channel=0)  # every rank is done with the buffer's previous contents
    common = (ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(ov), exact_blocks, scale_value,
              -2 if sink_block is None else sink_block, _lib.STATS_HYD, 1, full.data_ptr(),
              full.numel() * full.element_size())
    if use_multicast:
        _lib.check(_lib.LIB.b2_pisa_forward_multicast(*common, multicast, _lib.ptr(ws), _lib.stream_of(q)))
    else:
        _lib.check(_lib.LIB.b2_pisa_forward_mirrored(*common, mirrors, len(peers), _lib.ptr(ws), _lib.stream_of(q)))
    handle.barrier(channel=1)  # every rank's rows have landed in every copy
    if out is not None:
        out.copy_(full)
        return out
    return full
