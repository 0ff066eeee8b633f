"""Multi-process host logic of bench.py on CPU: two gloo ranks.

bench.py runs one process per GPU (strong scaling: the heads of one call
are split over the ranks and the outputs all-gathered); the host-side
cross-rank steps are the max over ranks of the timed region, the job value
and rank-0-only output.  Those run here with the gloo backend on
127.0.0.1, without a GPU (the head exchange itself: test_host_sharded.py).
"""
import io
import os
import pathlib
import socket
import sys
from contextlib import redirect_stdout

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, r, local = bench._dist()
        ms = 1.0 + rank  # rank 1 is the slow one
        slowest = bench.max_over_ranks(ms, torch.device("cpu"))
        value = bench.job_value(w, slowest)
        # the reference arm runs on rank 0 only; other ranks print nothing
        buf = io.StringIO()
        if rank != 0:
            args = type("A", (), {"warmup": 0, "steps": 0})()
            with redirect_stdout(buf):
                bench.run_reference(args)
        results[rank] = (w, r, local, slowest, value, buf.getvalue())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_slowest_time():
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    sys.path.insert(0, str(ROOT))
    import bench

    for rank in range(world):
        w, r, local, slowest, value, out = results[rank]
        assert (w, r, local) == (world, rank, rank)
        assert slowest == 2.0  # max over ranks, seen identically by every rank
        # strong scaling: the ranks share one call, timed by the slowest rank
        assert abs(value - bench.DENSE_FLOP / 2e-3 / 1e12) < 1e-9
        assert out == ""


def test_single_process_needs_no_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(3.5, torch.device("cpu")) == 3.5
    assert abs(bench.job_value(1, 1.0) - bench.DENSE_FLOP / 1e-3 / 1e12) < 1e-9


def test_secondary_workloads_count_the_configs_work():
    """Algorithmic work of the non-headline configs: dense flops 4*B*H*Tq*Tk*D
    (configs 2, 4, 5) and the FP32 fixed-block call (config 1)."""
    sys.path.insert(0, str(ROOT))
    import bench

    gflop = {name: make().value_work / 1e9 for name, make in bench.WORKLOADS.items()}
    assert round(gflop["full_self"], 1) == 1391.6
    assert round(gflop["full_cross"], 1) == 77.3
    assert round(gflop["minimax_h3_t9170"], 1) == 2411.0
    assert round(gflop["minimax_h3_t16500"], 1) == 7806.0
    assert round(gflop["generic_pisa_video"], 1) == 21979.5
    assert round(gflop["fixed_block_fp32"], 3) == 0.134
    generic = bench.WORKLOADS["generic_pisa_video"]()
    assert (generic.nb, generic.exact) == (512, 86)
    assert round(generic.roof_work / 1e9) == round(40 * 32760 * 86 * 4 * 64 * 128 / 1e9 + 4 * 40 * 32760 * 512 * 128 / 1e9
                                                   + 2 * 40 * 32760 * 128 * 128 / 1e9)
    assert bench.WORKLOADS["fixed_block_fp32"]().flush
    layout = bench.WORKLOADS["anima_layout_kernels"]()
    mb = 2 * 16 * 9216 * 128 * 2 / 1e6  # one [B,H,T,D] bf16 tensor
    assert abs(layout.pack_bytes / 1e6 - 6 * mb) < 1e-6            # q, k, v read + written
    assert abs(layout.unpack_bytes / 1e6 - 2 * mb) < 1e-6
    assert round(layout.merge_bytes / 1e6, 1) == 379.8             # 304.3 read + 75.5 written


def test_secondary_workload_reference_arm_prints_one_line():
    """The reference arm of a secondary config runs the oracle on host cores
    and prints the contract's line (impl, e2e with zero copy bytes,
    cpu_baseline describing the same run)."""
    import json

    sys.path.insert(0, str(ROOT))
    import bench

    args = type("A", (), {"warmup": 1, "steps": 2})()
    buf = io.StringIO()
    with redirect_stdout(buf):
        bench.run_workload_reference(args, bench.WORKLOADS["fixed_block_fp32"]())
    lines = [ln for ln in buf.getvalue().splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["config"]["workload"] == "fixed_block_fp32"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"] > 0
    assert line["unit"] == "GFLOP/s" and line["higher_is_better"] is True


def test_host_memory_call_rejects_pageable_buffers():
    import pytest

    sys.path.insert(0, str(ROOT / "comfyui-rdna35-attention_b200"))
    import b200_pisa

    x = torch.zeros((1, 9216, 2, 128), dtype=torch.bfloat16).permute(0, 2, 1, 3)
    with pytest.raises(ValueError, match="pinned"):
        b200_pisa.forward_spatial_bhtd_host(x, x, x, exact_blocks=23)
