"""Head-sharded PISA across the GPUs of one node.

Every (batch, head) of a PISA call is independent: the statistics, routing
and attention of one head never read another head's data (the reference's
kernels grid over batch*heads, native/rdna35_pisa_ck/csrc/pisa_kernels.cu:583,
and its FlexAttention call is per (batch, head)).  A call over H heads on N
GPUs (one process per GPU, torch.distributed with NCCL) therefore splits the
heads into N contiguous ranges: each rank computes its range with the
single-GPU kernels, then one NCCL all-gather exchanges the outputs over
NVLink, and a 16-byte copy kernel interleaves the gathered [N,B,T,Hs*D]
shards into the caller's [B,T,H*D] raster.  Because a head's output does
not depend on which other heads share its call, the sharded result equals
the single-GPU result bit for bit.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


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


def forward_spatial_bhtd_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                                 scale: float | None = None, sink_block: int | None = None, *, group=None,
                                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Anima spatial PISA over the heads of all ranks of `group`.

    q/k/v: this rank's head shard, BHTD views [B,Hs,9216,128] of contiguous
    [B,9216,Hs,128] BF16 storage (heads head_range(H, N, rank) of the full
    call).  Returns the full [B,9216,N*Hs*128] raster output on every rank,
    equal to forward_spatial_bhtd over all H heads on one GPU."""
    from . import forward_spatial_bhtd

    local = forward_spatial_bhtd(q, k, v, exact_blocks, scale=scale, sink_block=sink_block)
    return gather_head_shards(local, group=group, out=out)
