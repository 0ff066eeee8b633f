"""One rank of the multi-GPU head-sharding check (run under torchrun by
tests/test_gpu_multi.py): every rank computes its heads of the config-3
call with the default (peer-store) exchange, the multicast exchange where
the system offers it, and the NCCL exchange, and every result is compared with the
single-GPU call over all heads, bit for bit."""
import os
import pathlib
import sys

import torch
import torch.distributed as dist

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT / "comfyui-rdna35-attention_b200", ROOT / "oracle"):
    sys.path.insert(0, str(p))


def has_multicast() -> bool:
    from b200_pisa import sharded

    return any(getattr(h, "multicast_ptr", 0) for _, h in sharded._SYMMETRIC.values())


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import b200_pisa
    import pisa_oracle
    from b200_pisa.sharded import forward_spatial_bhtd_sharded, head_range

    world, rank = dist.get_world_size(), dist.get_rank()
    q, k, v = pisa_oracle.anima_inputs(batch=2, heads=16, seed=77)
    h0, h1 = head_range(16, world, rank)
    shard = [x[:, h0:h1].permute(0, 2, 1, 3).contiguous().cuda().permute(0, 2, 1, 3) for x in (q, k, v)]
    ok = True
    for _ in range(2):  # twice: the symmetric buffer is reused
        auto = forward_spatial_bhtd_sharded(*shard, 23).clone()
        multi = forward_spatial_bhtd_sharded(*shard, 23, exchange="multicast").clone() if has_multicast() else auto
        peer = forward_spatial_bhtd_sharded(*shard, 23, exchange="peer").clone()
        nccl = forward_spatial_bhtd_sharded(*shard, 23, exchange="nccl")
        torch.cuda.synchronize()
        full = [x.permute(0, 2, 1, 3).contiguous().cuda().permute(0, 2, 1, 3) for x in (q, k, v)]
        ref = b200_pisa.forward_spatial_bhtd(*full, 23)
        ok = ok and torch.equal(auto, ref) and torch.equal(multi, ref) and torch.equal(peer, ref) and torch.equal(nccl, ref)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        from b200_pisa import sharded
        _, handle = next(iter(sharded._SYMMETRIC.values()))
        print("multicast:", bool(getattr(handle, "multicast_ptr", 0)))
        print("SHARDED_OK" if flag.item() == 1 else "SHARDED_MISMATCH")
    dist.destroy_process_group()
    return 0 if flag.item() == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
