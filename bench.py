"""Benchmark of the B200 PISA attention call (BASELINE.json metric).

Workload: Anima PISA HYD spatial self-attention,
BF16 q/k/v [B=2,H=16,T=9216,D=128] as BHTD views of raster [B,T,H,D]
storage, 23 of 144 exact KV blocks per query block.  One step = one
``b200_pisa.forward_spatial_bhtd`` call over the whole batch (statistics,
routing, fused exact + tail + correction attention, raster output).

Multi-GPU (torchrun, one process per GPU): strong scaling of the same call --
the 16 heads are split into N equal contiguous ranges
(``b200_pisa.sharded.head_range``); each rank holds its heads' q/k/v
([B,T,H/N,D] raster) and computes them with the single-GPU kernels, and the
full [B,T,H*D] output is assembled on every rank
(``forward_spatial_bhtd_sharded``: the attention epilogue stores each output
row into every rank's copy of a symmetric output buffer over NVLink; the
NCCL all-gather + interleave variant is timed beside it).  Timing: W untimed warm-ups,
then K steps between a barrier + synchronize on both sides, CUDA events on
the launching stream, max over ranks.  The inputs (226 MB of q/k/v) exceed
the 126 MB L2, so no extra flush.

``e2e`` is the same call for activations in pinned host memory.  On one GPU
it is ``b200_pisa.forward_spatial_bhtd_host`` (the copies in and out are
inside the timed region and overlap the compute of neighbouring head
stages; the unstaged copy-in, call, copy-out time is reported beside it).
On N GPUs each rank copies its heads' q/k/v in, runs the sharded call and
copies its heads' columns of the output out (the job's input and output
each cross PCIe once; the line gives per-rank and job byte counts).

``--impl reference`` times the reference's PyTorch HYD path restated on the
host CPU (oracle/pisa_oracle.py, the batched form that mirrors the
reference's torch ops) for the whole 32-head call and reports the same
metric.

``--workload`` selects one of the other configs instead of the headline one
(full_self / full_cross: config 2; minimax_h3_t9170 / minimax_h3_t16500:
config 4; generic_pisa_video: config 5; fixed_block_fp32: config 1;
anima_layout_kernels: the standalone pack / unpack / merge kernels of
config 3).  Each
prints the same JSON line for its own public call, with the roofline of its
dominant kernel and a bounded CPU sample of the oracle.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import time

import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "comfyui-rdna35-attention_b200"))

B, H, T, D = 2, 16, 9216, 128
NB = T // 64
EXACT = 23
METRIC = "PISA attn call ms & dense-equiv TFLOP/s, B=2 H=16 T=9216 D=128 bf16"
UNIT = "dense-equiv TFLOP/s"
DENSE_FLOP = 4.0 * B * H * T * T * D                     # 1391.6 GFLOP per call
EXACT_FLOP = 4.0 * B * H * NB * EXACT * 64 * 64 * D       # 222.3 GFLOP
TAIL_FLOP = 4.0 * B * H * T * NB * D                      # 21.7 GFLOP (q.kc and p.vc)
CORR_FLOP = 2.0 * B * H * T * D * D                       # 9.66 GFLOP
STATS_BYTES = 3 * B * H * T * D * 2                       # q/k/v read once
# dram__bytes_read.sum + dram__bytes_write.sum per launch from one ncu
# capture of this workload's attention and statistics kernels
ATTN_TRAFFIC = 288.8e6
STATS_TRAFFIC = 240.2e6
CONFIG = {
    "workload": "anima_pisa_hyd_spatial",
    "batch": B, "heads": H, "tokens": T, "head_dim": D, "exact_blocks": EXACT, "blocks": NB,
    "layout": "BHTD views of raster [B,T,H,D]; output [B,T,H*D]",
    "l2": "inputs 226 MB > 126 MB L2 (no flush)",
}


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm": data["hbm_gbs"], "bf16": data["bf16_tflops"], "bf16_sustained": data.get("bf16_tflops_sustained"),
                "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, device) -> float:
    """The slowest rank's time: all-reduce MAX over the process group (NCCL
    on the GPUs, gloo in the CPU tests); the value itself with one rank."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_value(world: int, ms: float) -> float:
    """Whole-job dense-equivalent TFLOP/s: the N ranks together run one
    config-3 call (strong scaling: heads split over the ranks, outputs
    gathered), which takes the slowest rank's time."""
    del world  # the call's work does not grow with the number of ranks
    return DENSE_FLOP / (ms * 1e-3) / 1e12


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.path = pathlib.Path(os.environ.get("TMPDIR", "/tmp")) / f"b2_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


def _inputs(device, seed):
    import pisa_oracle

    q, k, v = pisa_oracle.anima_inputs(batch=B, heads=H, seed=seed)
    return q, k, v


def _graph_timed(fn, steps, stream):
    """Device time of `fn` from a CUDA graph of `steps` back-to-back calls
    (removes the host launch gaps that dominate short kernels)."""
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    graph.replay()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps


def _timed(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps


def run_b200(args) -> None:
    world, rank, local = _dist()
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sys.path.insert(0, str(ROOT / "oracle"))
    import b200_pisa
    from b200_pisa import _lib
    from b200_pisa.sharded import forward_spatial_bhtd_sharded, gather_head_shards, head_range

    b200_pisa.prepare(local)
    h0, h1 = head_range(H, world, rank)
    hs = h1 - h0
    q_cpu, k_cpu, v_cpu = _inputs(device, seed=0)  # the same call on every rank
    # this rank's heads as raster BTHD storage on the host (pinned), BHTD views on the device
    host = [x[:, h0:h1].permute(0, 2, 1, 3).contiguous().pin_memory() for x in (q_cpu, k_cpu, v_cpu)]
    del q_cpu, k_cpu, v_cpu
    dev = [h.to(device).permute(0, 2, 1, 3) for h in host]
    q, k, v = dev
    stream = torch.cuda.current_stream(device)
    out_dev = torch.empty((B, T, H * D), device=device, dtype=torch.bfloat16)

    def step():
        if world == 1:
            return b200_pisa.forward_spatial_bhtd(q, k, v, exact_blocks=EXACT)
        return forward_spatial_bhtd_sharded(q, k, v, EXACT)  # peer-store exchange

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(device)

    if args.profile_only:
        # launch-list / ncu mode: warm-ups + K plain steps, nothing else
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize(device)
        print(json.dumps({"profile_only": True, "steps": args.steps, "warmup": args.warmup}))
        return
    with ClockSampler(local) as clocks:
        barrier()
        ms = _timed(step, args.steps, stream)
        barrier()
    clock_info = clocks.summary()
    ms = max_over_ranks(ms, device)
    value = job_value(world, ms)
    gather_ms = nccl_ms = None
    if world > 1:
        # the alternative exchange: local call, NCCL all-gather + interleave
        local_out = b200_pisa.forward_spatial_bhtd(q, k, v, exact_blocks=EXACT)
        barrier()
        gather_ms = max_over_ranks(_timed(lambda: gather_head_shards(local_out, out=out_dev), args.steps, stream),
                                   device)
        barrier()
        nccl_ms = max_over_ranks(_timed(lambda: forward_spatial_bhtd_sharded(q, k, v, EXACT, out=out_dev,
                                                                             exchange="nccl"), args.steps, stream),
                                 device)
        barrier()

    # ---- end to end through the public API for host-resident activations
    out_host = torch.empty((B, T, H * D), dtype=torch.bfloat16).pin_memory()
    host_bhtd = [h.permute(0, 2, 1, 3) for h in host]
    serial_ms = None
    if world == 1:
        # pinned host q/k/v in, pinned host output out, all inside the timed
        # region; forward_spatial_bhtd_host stages the call by heads so the
        # PCIe copies overlap the compute of neighbouring stages
        def e2e_step():
            b200_pisa.forward_spatial_bhtd_host(*host_bhtd, exact_blocks=EXACT, device=device, out=out_host,
                                                heads_per_stage=args.heads_per_stage)
    else:
        # this rank's heads in, sharded call (every rank then holds the full
        # output), and this rank's share of the job's output back to the host:
        # its heads' columns, so the job's result crosses PCIe once in total
        dev_bthd = [torch.empty_like(h, device=device) for h in host]
        out_host = torch.empty((B, T, hs * D), dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            for d_, h_ in zip(dev_bthd, host):
                d_.copy_(h_, non_blocking=True)
            out = forward_spatial_bhtd_sharded(*(x.permute(0, 2, 1, 3) for x in dev_bthd), EXACT)
            out_host.copy_(out[:, :, h0 * D:h1 * D], non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    e2e_ms = _timed(e2e_step, max(2, args.steps // 2), stream)
    barrier()
    e2e_ms = max_over_ranks(e2e_ms, device)

    if world == 1:
        # the same end-to-end call without staging (copy all in, call, copy out)
        dev_bthd = [torch.empty_like(h, device=device) for h in host]

        def serial_step():
            for d_, h_ in zip(dev_bthd, host):
                d_.copy_(h_, non_blocking=True)
            out = b200_pisa.forward_spatial_bhtd(*(x.permute(0, 2, 1, 3) for x in dev_bthd), exact_blocks=EXACT)
            out_host.copy_(out, non_blocking=True)

        serial_step()
        barrier()
        serial_ms = max_over_ranks(_timed(serial_step, max(2, args.steps // 4), stream), device)
        barrier()
        del dev_bthd
    h2d = sum(h.numel() * h.element_size() for h in host)
    d2h = out_host.numel() * out_host.element_size()

    # ---- component timing (dominant kernels, separate entry points, this rank's heads)
    comp = component_times(b200_pisa, _lib, q, k, v, device, stream, args.steps)

    peaks = _peaks()
    share = hs / H
    attn_flop = (EXACT_FLOP + TAIL_FLOP + CORR_FLOP) * share
    achieved = attn_flop / (comp["attention_ms"] * 1e-3) / 1e12
    stats_gbs = STATS_BYTES * share / (comp["stats_ms"] * 1e-3) / 1e9
    roofline = {
        "kernel": "attn_kernel (fused exact + tail + correction)",
        "bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16"], "unit": "TFLOP/s",
        "frac": round(achieved / peaks["bf16"], 4), "peak_source": peaks["source"] + " bf16 burst",
        "traffic": (args.traffic if args.traffic is not None else ATTN_TRAFFIC) * share,
        "stats_kernel": {
            "bound": "hbm", "achieved": round(stats_gbs, 1), "peak": peaks["hbm"], "unit": "GB/s",
            "frac": round(stats_gbs / peaks["hbm"], 4), "traffic": STATS_TRAFFIC * share,
        },
        "component_ms": comp,
    }
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) + per-tile N(0,0.5) offsets)",
            "config": {**CONFIG, "parallelism": f"heads split over {world} GPU(s), {hs} per rank"
                       + (", outputs exchanged by peer stores from the attention epilogue" if world > 1 else "")},
            "clocks": clock_info,
            "e2e": {"value": round(job_value(world, e2e_ms), 2), "unit": UNIT,
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    **({"bytes_per_rank": True, "job_h2d_bytes_per_step": h2d * world,
                        "job_d2h_bytes_per_step": d2h * world} if world > 1 else {}),
                    "api": "forward_spatial_bhtd_host" if world == 1 else "forward_spatial_bhtd_sharded",
                    **({"heads_per_stage": args.heads_per_stage, "unstaged_ms_per_step": round(serial_ms, 4)}
                       if world == 1 else {})},
            "gpu_launches": 6 * args.steps,
            "roofline": roofline,
        }
        if gather_ms is not None:
            line["nccl_exchange"] = {"call_ms": round(nccl_ms, 4), "all_gather_and_interleave_ms": round(gather_ms, 4)}
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def component_times(b200_pisa, _lib, q, k, v, device, stream, steps):
    """Time the statistics kernel and the fused attention kernel separately
    through their own C-ABI entry points (same buffers as the full call)."""
    import ctypes

    from b200_pisa import LIB, check

    heads = q.shape[1]
    bh = B * heads
    grid = dict(order=_lib.ORDER_TILED8, grid=(96, 96))
    qv, kv, vv = (_lib.view(x, **grid) for x in (q, k, v))
    out = torch.empty((B, T, heads * D), device=device, dtype=torch.bfloat16)
    ov = _lib.view(out.view(B, T, heads, D).permute(0, 2, 1, 3), **grid)
    qc = torch.empty((bh, NB, D), device=device, dtype=torch.bfloat16)
    kc = torch.empty((bh, NB, D), device=device, dtype=torch.float32)
    vc = torch.empty((bh, NB, D), device=device, dtype=torch.bfloat16)
    hs = torch.empty((bh, D, D), device=device, dtype=torch.float32)
    hn = torch.empty((bh, NB), device=device, dtype=torch.float32)
    h16 = torch.empty((bh, D, D), device=device, dtype=torch.bfloat16)
    ws = torch.empty(int(LIB.b2_stats_workspace_bytes(bh, T, D)), device=device, dtype=torch.uint8)
    idx = torch.empty((bh, NB, EXACT), device=device, dtype=torch.int32)
    sel = torch.empty((bh, NB, (NB + 31) // 32), device=device, dtype=torch.int32)
    nonlocal_streams = [stream.cuda_stream]
    scale = 1.0 / math.sqrt(D)

    def stats():
        check(LIB.b2_pisa_block_stats(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), _lib.STATS_HYD,
                                      qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), hs.data_ptr(), hn.data_ptr(),
                                      h16.data_ptr(), ws.data_ptr(), nonlocal_streams[0]))

    def route():
        check(LIB.b2_pisa_route(qc.data_ptr(), _lib.B2_BF16, kc.data_ptr(), _lib.B2_BF16, hn.data_ptr(), bh, NB, D,
                                EXACT, scale, -2, idx.data_ptr(), sel.data_ptr(), nonlocal_streams[0]))

    kc16 = kc.to(torch.bfloat16)
    pairs = torch.empty((bh, (NB + 1) // 2, 2), device=device, dtype=torch.int32)

    def pair():
        check(LIB.b2_pisa_pair(sel.data_ptr(), bh, NB, pairs.data_ptr(), nonlocal_streams[0]))

    def attn():
        check(LIB.b2_pisa_attention(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(ov),
                                    idx.data_ptr(), EXACT, sel.data_ptr(), pairs.data_ptr(), kc16.data_ptr(),
                                    vc.data_ptr(), h16.data_ptr(), scale, None, nonlocal_streams[0]))

    stats()
    route()
    pair()
    kc16.copy_(kc.to(torch.bfloat16))
    for fn in (stats, route, pair, attn):
        fn()
    torch.cuda.synchronize(device)
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        st_side = side.cuda_stream
        nonlocal_streams[0] = st_side
        out = {name: round(_graph_timed(fn, steps, side), 4)
               for name, fn in (("stats_ms", stats), ("route_ms", route), ("pair_ms", pair), ("attention_ms", attn))}
    nonlocal_streams[0] = stream.cuda_stream
    torch.cuda.synchronize(device)
    return out


def _oracle_call(q, k, v):
    """The reference's HYD path restated on the host (oracle/pisa_oracle.py,
    batched form of rdna35_pisa_ck/__init__.py:254-316): pack, statistics,
    routing, gathered exact + tail + correction, raster output."""
    import pisa_oracle

    packed = [pisa_oracle.pack_spatial(x) for x in (q, k, v)]
    out, _ = pisa_oracle.hyd_forward_batched(*packed, EXACT)
    return pisa_oracle.unpack_spatial(out, q.shape[0], q.shape[1])


def cpu_baseline() -> dict:
    """The oracle on all host cores, one full 32-head call (a few seconds)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v = _inputs(None, seed=0)
    t0 = time.perf_counter()
    _oracle_call(q, k, v)
    sec = time.perf_counter() - t0
    return {"value": round(DENSE_FLOP / sec / 1e12, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"one full call, all {B * H} (batch, head) pairs at T=9216 (no extrapolation)",
            "ms_per_call": round(sec * 1e3, 1)}


def run_reference(args) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v = _inputs(None, seed=0)
    for _ in range(args.warmup):
        _oracle_call(q, k, v)
    samples = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _oracle_call(q, k, v)
        samples.append(time.perf_counter() - t0)
    call_ms = statistics.median(samples) * 1e3
    value = DENSE_FLOP / (call_ms * 1e-3) / 1e12
    sample = f"one full call per step, all {B * H} (batch, head) pairs at T=9216 (no extrapolation)"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(call_ms, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": CONFIG,
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------- other configs
# The other BASELINE.json configs, each timed through its public call under
# the same JSON contract (``--workload``).  Config 3 ("anima") stays the
# headline line; these are reported beside it.


def _randn(shape, gen, dtype=torch.bfloat16):
    return torch.randn(shape, generator=gen).to(dtype)


class Workload:
    """One secondary config: host inputs, the public call on device views,
    the roofline of its dominant kernel, and a bounded CPU sample."""

    def __init__(self, name, config, metric, unit, value_work, roof_bound, roof_work, launches, flush=False):
        self.name, self.config, self.metric, self.unit = name, config, metric, unit
        self.value_work, self.roof_bound, self.roof_work = value_work, roof_bound, roof_work
        self.launches, self.flush = launches, flush
        self.value_scale = 1e9 if unit.startswith(("GFLOP", "GB")) else 1e12

    # subclasses: host_inputs(seed) -> list of CPU tensors; views(dev) -> call
    # arguments; call(api, *args) -> output; kernel(api, *args) -> a callable
    # timing the dominant kernel alone; cpu_call() -> (seconds per full call,
    # sample text)


class FullWorkload(Workload):
    """Config 2: exact full attention, self (Tk=9216) or cross (Tk=512)."""

    def __init__(self, tk):
        flop = 4.0 * B * H * T * tk * D
        name = "full_self" if tk == T else "full_cross"
        super().__init__(name, {"workload": name, "batch": B, "heads": H, "q_tokens": T, "kv_tokens": tk,
                                "head_dim": D, "layout": "contiguous [B,H,T,D]",
                                "l2": "q/out 151 MB > 126 MB L2 (no flush)"},
                         f"full attention call ms & TFLOP/s, B=2 H=16 Tq=9216 Tk={tk} D=128 bf16", "TFLOP/s",
                         flop, "tensor", flop, 1)
        self.tk = tk

    def host_inputs(self, seed):
        gen = torch.Generator().manual_seed(seed)
        return [_randn((B, H, T, D), gen), _randn((B, H, self.tk, D), gen), _randn((B, H, self.tk, D), gen)]

    def views(self, dev):
        return dev

    def call(self, api, q, k, v):
        return api.full_attention(q, k, v, D ** -0.5)

    def cpu_call(self):
        import pisa_oracle

        if not hasattr(self, "_cpu"):
            self._cpu = self.host_inputs(0)
        q, k, v = self._cpu
        t0 = time.perf_counter()
        pisa_oracle.full_attention(q[0, :1], k[0, :1], v[0, :1])
        return (time.perf_counter() - t0) * B * H, f"1 of {B * H} (batch, head) pairs, scaled x{B * H}"


class H3Workload(Workload):
    """Config 4: MiniMax-H3 exact attention from the interleaved projection
    [1,T,3,56,128]; q/k are strided views, v a contiguous clone viewed BHTD
    (bench_minimax_h3_gfx1151_attention.py:90-94).  One call = the override's
    native path (attention straight from the views + merged [B,T,H*D] output;
    no pack copy is needed)."""

    HEADS = 56

    def __init__(self, tokens):
        flop = 4.0 * self.HEADS * tokens * tokens * D
        name = f"minimax_h3_t{tokens}"
        super().__init__(name, {"workload": name, "batch": 1, "heads": self.HEADS, "tokens": tokens, "head_dim": D,
                                "layout": "q,k strided views of qkv [1,T,3,56,128]; v contiguous; out [1,T,56*128]",
                                "l2": "inputs > 126 MB L2 (no flush)"},
                         f"MiniMax-H3 attention call ms & TFLOP/s, H=56 T={tokens} D=128 bf16", "TFLOP/s",
                         flop, "tensor", flop, 1)
        self.tokens = tokens

    def host_inputs(self, seed):
        gen = torch.Generator().manual_seed(self.tokens if seed == 0 else self.tokens + seed)
        qkv = _randn((1, self.tokens, 3, self.HEADS, D), gen)
        return [qkv, qkv[:, :, 2].contiguous()]

    def views(self, dev):
        qkv, v = dev
        return qkv[:, :, 0].permute(0, 2, 1, 3), qkv[:, :, 1].permute(0, 2, 1, 3), v.permute(0, 2, 1, 3)

    def call(self, api, q, k, v):
        from rdna35_block_attention.minimax_h3_gfx1151_attention import minimax_h3_attention

        return minimax_h3_attention(q, k, v)

    def cpu_call(self):
        import pisa_oracle

        if not hasattr(self, "_cpu"):
            self._cpu = self.host_inputs(0)
        qkv, v = self._cpu
        q, k = qkv[:, :, 0, :1].permute(0, 2, 1, 3), qkv[:, :, 1, :1].permute(0, 2, 1, 3)
        t0 = time.perf_counter()
        pq, pk, pv, _ = pisa_oracle.h3_pack(q, k, v[:, :, :1].permute(0, 2, 1, 3))
        pisa_oracle.full_attention(pq, pk, pv)
        return (time.perf_counter() - t0) * self.HEADS, f"1 of {self.HEADS} heads (pack + attention), scaled x56"


class GenericWorkload(Workload):
    """Config 5: generic PISA video self-attention [1,40,32760,128], 512
    blocks (last 56 tokens), ceil(512/6) = 86 exact, first-order on."""

    HEADS, TOKENS = 40, 32760

    def __init__(self):
        nb = (self.TOKENS + 63) // 64
        self.nb, self.exact = nb, math.ceil(nb / 6)
        exact = 4.0 * self.HEADS * self.TOKENS * 64 * self.exact * D  # every row x 86 selected 64-key blocks
        tail = 4.0 * self.HEADS * self.TOKENS * nb * D
        corr = 2.0 * self.HEADS * self.TOKENS * D * D
        dense = 4.0 * self.HEADS * self.TOKENS * self.TOKENS * D
        super().__init__("generic_pisa_video", {"workload": "generic_pisa_video", "batch": 1, "heads": self.HEADS,
                                                "tokens": self.TOKENS, "head_dim": D, "blocks": nb,
                                                "exact_blocks": self.exact, "layout": "block-major [1,40,T,128]",
                                                "l2": "inputs 1.0 GB > 126 MB L2 (no flush)"},
                         "generic PISA call ms & dense-equiv TFLOP/s, H=40 T=32760 D=128 bf16, 86/512 exact",
                         "dense-equiv TFLOP/s", dense, "tensor", exact + tail + corr, 5)

    def host_inputs(self, seed):
        import pisa_oracle

        q, k, v = pisa_oracle.generic_inputs(self.HEADS, self.TOKENS, seed)
        return [x.unsqueeze(0) for x in (q, k, v)]

    def _cpu_inputs(self):
        if not hasattr(self, "_cpu"):
            import pisa_oracle

            self._cpu = pisa_oracle.generic_inputs(1, self.TOKENS, 0)
        return self._cpu

    def views(self, dev):
        return dev

    def call(self, api, q, k, v):
        return api.generic_forward(q, k, v, self.exact, D ** -0.5)

    def kernel(self, api, q, k, v):
        """The fused attention launch alone, fed by this call's own statistics,
        routing and pairing (C-ABI entry points); the other stages are
        returned beside it for their own timings."""
        import ctypes

        from b200_pisa import LIB, _lib, check

        bh, nb, dev = self.HEADS, self.nb, q.device
        stream = lambda: torch.cuda.current_stream(dev).cuda_stream  # noqa: E731
        qv, kv, vv = (_lib.view(x) for x in (q, k, v))
        qc = torch.empty((bh, nb, D), device=dev, dtype=torch.float32)
        kc = torch.empty_like(qc)
        vsum = torch.empty_like(qc)
        hsum = torch.empty((bh, D, D), device=dev, dtype=torch.float32)
        ws = torch.empty(int(LIB.b2_stats_workspace_bytes(bh, self.TOKENS, D)), device=dev, dtype=torch.uint8)
        idx = torch.empty((bh, nb, self.exact), device=dev, dtype=torch.int32)
        sel = torch.empty((bh, nb, (nb + 31) // 32), device=dev, dtype=torch.int32)
        pairs = torch.empty((bh, (nb + 1) // 2, 2), device=dev, dtype=torch.int32)

        def stats():
            check(LIB.b2_pisa_block_stats(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), _lib.STATS_GENERIC,
                                          qc.data_ptr(), kc.data_ptr(), vsum.data_ptr(), hsum.data_ptr(), None, None,
                                          ws.data_ptr(), stream()))

        def route():
            check(LIB.b2_pisa_route(qc.data_ptr(), _lib.B2_F32, kc.data_ptr(), _lib.B2_F32, None, bh, nb, D,
                                    self.exact, D ** -0.5, -2, idx.data_ptr(), sel.data_ptr(), stream()))

        def pair():
            check(LIB.b2_pisa_pair(sel.data_ptr(), bh, nb, pairs.data_ptr(), stream()))

        stats()
        route()
        pair()
        lens = torch.full((nb,), 64.0, device=dev)
        lens[-1] = self.TOKENS - 64 * (nb - 1)
        kc16 = kc.to(torch.bfloat16)
        vc16 = (vsum / lens[None, :, None]).to(torch.bfloat16)
        h16 = hsum.to(torch.bfloat16)
        out = torch.empty_like(q)
        ov = _lib.view(out)

        def attn():
            check(LIB.b2_pisa_attention(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(ov),
                                        idx.data_ptr(), self.exact, sel.data_ptr(), pairs.data_ptr(), kc16.data_ptr(),
                                        vc16.data_ptr(), h16.data_ptr(), D ** -0.5, None, stream()))

        # the views hold raw pointers: the tensors behind them must outlive
        # every launch (CUDA-graph capture empties the allocator's cache)
        attn.keep_alive = (q, k, v, out, qc, kc, vsum, hsum, ws, idx, sel, pairs, kc16, vc16, h16)
        attn.components = {"stats_ms": stats, "route_ms": route, "pair_ms": pair}
        return attn

    def cpu_call(self):
        import pisa_oracle

        q, k, v = self._cpu_inputs()
        t0 = time.perf_counter()
        pisa_oracle.generic_forward(q, k, v, self.exact)
        return (time.perf_counter() - t0) * self.HEADS, f"1 of {self.HEADS} heads at T=32760, scaled x40"


class FixedWorkload(Workload):
    """Config 1: fixed 64-token block-diagonal attention, FP32 [1,8,1024,64]."""

    def __init__(self):
        self.shape = (1, 8, 1024, 64)
        flop = 4.0 * 8 * 1024 * 64 * 64
        nbytes = 4.0 * 4 * 8 * 1024 * 64
        super().__init__("fixed_block_fp32", {"workload": "fixed_block_fp32", "batch": 1, "heads": 8, "tokens": 1024,
                                              "head_dim": 64, "block": 64,
                                              "l2": "8.4 MB inputs: L2 flushed (256 MB write) before every step"},
                         "fixed-block attention call ms & GFLOP/s, B=1 H=8 T=1024 D=64 fp32", "GFLOP/s",
                         flop, "hbm", nbytes, 1, flush=True)

    def host_inputs(self, seed):
        gens = [torch.Generator().manual_seed(s) for s in (0 + 3 * seed, 1 + 3 * seed, 2 + 3 * seed)]
        return [torch.randn(self.shape, generator=g) for g in gens]

    def views(self, dev):
        return dev

    def call(self, api, q, k, v):
        from rdna35_block_attention.dispatch import fixed_block_attention

        return fixed_block_attention(q, k, v, mode="b200")

    def kernel(self, api, q, k, v):
        """The FP32 block-diagonal launch alone through its C-ABI entry."""
        import ctypes

        from b200_pisa import LIB, _lib, check

        out = torch.empty_like(q)
        qv, kv, vv, ov = (_lib.view(x) for x in (q, k, v, out))

        def fixed():
            check(LIB.b2_fixed_block_attention(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv),
                                               ctypes.byref(ov), ctypes.c_float(0.125), 0,
                                               ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)))

        fixed.keep_alive = (q, k, v, out)
        return fixed

    def cpu_call(self):
        import pisa_oracle

        q, k, v = self.host_inputs(0)
        reps = 50
        t0 = time.perf_counter()
        for _ in range(reps):
            pisa_oracle.fixed_block_attention(q, k, v)
        return (time.perf_counter() - t0) / reps, f"the whole config, mean of {reps} calls"


class LayoutWorkload(Workload):
    """The standalone layout kernels of the Anima path that the reference's
    `_C` module exposes (rows a2, a8, a9): raster -> block-major pack of
    q/k/v (the call), block-major -> raster unpack and the LSE-weighted merge
    epilogue (components).  All three are HBM copies; the fused PISA call
    does not run them."""

    def __init__(self):
        row = B * H * T * D * 2
        self.pack_bytes = 3.0 * 2 * row                           # 3 x (75.5 MB read + write)
        self.unpack_bytes = 2.0 * row                             # 75.5 MB read + write
        self.merge_bytes = 2.0 * row + 4.0 * B * H * T * D + 2 * 4.0 * B * H * T + row  # 304.3 + 75.5 MB
        super().__init__("anima_layout_kernels", {"workload": "anima_layout_kernels", "batch": B, "heads": H,
                                                  "tokens": T, "head_dim": D,
                                                  "layout": "BHTD views of raster [B,T,H,D] <-> block-major [BH,T,D]",
                                                  "l2": "inputs 226 MB > 126 MB L2 (no flush)"},
                         "PISA spatial pack GB/s, B=2 H=16 T=9216 D=128 bf16", "GB/s", self.pack_bytes, "hbm",
                         self.pack_bytes, 3)

    def host_inputs(self, seed):
        import pisa_oracle

        return [x.permute(0, 2, 1, 3).contiguous() for x in pisa_oracle.anima_inputs(batch=B, heads=H, seed=seed)]

    def views(self, dev):
        return [x.permute(0, 2, 1, 3) for x in dev]

    def call(self, api, q, k, v):
        return api._C.pack_spatial_qkv(q, k, v)[0]

    def kernel(self, api, q, k, v):
        dev = q.device
        gen = torch.Generator(device=dev).manual_seed(5)
        bh = B * H
        blk = torch.randn((bh, T, D), generator=gen, device=dev).to(torch.bfloat16)
        approx = torch.randn((bh, T, D), generator=gen, device=dev).to(torch.bfloat16)
        corr = torch.randn((bh, T, D), generator=gen, device=dev)
        lse_e = torch.randn((bh, T), generator=gen, device=dev)
        lse_a = torch.randn((bh, T), generator=gen, device=dev)

        def pack():
            api._C.pack_spatial_qkv(q, k, v)

        def unpack():
            api._C.unpack_spatial_output(blk, B, H)

        def merge():
            api._C.fuse_spatial_epilogue(blk, lse_e, approx, lse_a, corr, B, H)

        pack.keep_alive = (q, k, v, blk, approx, corr, lse_e, lse_a)
        pack.components = {"unpack_ms": unpack, "merge_ms": merge}
        pack.component_bytes = {"unpack_ms": self.unpack_bytes, "merge_ms": self.merge_bytes}
        return pack

    def cpu_call(self):
        import pisa_oracle

        if not hasattr(self, "_cpu"):
            self._cpu = [x[:, :1] for x in pisa_oracle.anima_inputs(batch=1, heads=1, seed=0)]
        t0 = time.perf_counter()
        for x in self._cpu:
            pisa_oracle.pack_spatial(x)
        return (time.perf_counter() - t0) * B * H, f"1 of {B * H} (batch, head) pairs, scaled x{B * H}"


WORKLOADS = {
    "full_self": lambda: FullWorkload(T),
    "full_cross": lambda: FullWorkload(512),
    "minimax_h3_t9170": lambda: H3Workload(9170),
    "minimax_h3_t16500": lambda: H3Workload(16500),
    "generic_pisa_video": GenericWorkload,
    "fixed_block_fp32": FixedWorkload,
    "anima_layout_kernels": LayoutWorkload,
}


def _timed_flushed(fn, steps, stream, flush):
    """Mean device time of `fn` over `steps` calls, each after a write of a
    buffer twice the size of L2 (outside the timed events).  A short device
    sleep after the flush keeps the GPU busy while the host issues the step,
    so the events bracket device work, not host launch latency."""
    total = 0.0
    for _ in range(steps):
        flush.zero_()
        torch.cuda._sleep(400_000)  # ~0.2 ms of device time
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        fn()
        end.record(stream)
        end.synchronize()
        total += start.elapsed_time(end)
    return total / steps


def run_workload(args, wl) -> None:
    world, rank, local = _dist()
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sys.path.insert(0, str(ROOT / "oracle"))
    import b200_pisa as api

    api.prepare(local)
    host = [x.contiguous().pin_memory() for x in wl.host_inputs(rank)]
    dev = [h.to(device) for h in host]
    call_args = wl.views(dev)
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device) if wl.flush else None

    def step():
        return wl.call(api, *call_args)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(device)

    def timed(fn, steps):
        return _timed_flushed(fn, steps, stream, flush) if flush is not None else _timed(fn, steps, stream)

    with ClockSampler(local) as clocks:
        barrier()
        ms = timed(step, args.steps)
        barrier()
    clock_info = clocks.summary()
    ms = max_over_ranks(ms, device)
    value = world * wl.value_work / (ms * 1e-3) / wl.value_scale

    # end to end: pinned host inputs -> device, call, output -> pinned host
    sample_out = step()
    out_host = torch.empty(sample_out.shape, dtype=sample_out.dtype).pin_memory()
    dev_e2e = [torch.empty_like(h, device=device) for h in host]
    e2e_args = wl.views(dev_e2e)

    def e2e_step():
        for d_, h_ in zip(dev_e2e, host):
            d_.copy_(h_, non_blocking=True)
        out_host.copy_(wl.call(api, *e2e_args), non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    e2e_ms = max_over_ranks(timed(e2e_step, max(2, args.steps // 2)), device)
    barrier()

    # the dominant kernel alone (graph of back-to-back launches, or flushed)
    kernel = wl.kernel(api, *call_args) if hasattr(wl, "kernel") else step
    kernel()
    torch.cuda.synchronize(device)
    components = {}
    if flush is not None:
        kernel_ms = _timed_flushed(kernel, args.steps, stream, flush)
    else:
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            kernel_ms = _graph_timed(kernel, args.steps, side)
            for name, fn in getattr(kernel, "components", {}).items():
                components[name] = round(_graph_timed(fn, args.steps, side), 4)
        torch.cuda.synchronize(device)
    peaks = _peaks()
    if wl.roof_bound == "tensor":
        achieved, peak, unit = wl.roof_work / (kernel_ms * 1e-3) / 1e12, peaks["bf16"], "TFLOP/s"
    else:
        achieved, peak, unit = wl.roof_work / (kernel_ms * 1e-3) / 1e9, peaks["hbm"], "GB/s"
    if rank == 0:
        line = {
            "metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if wl.flush else "bf16", "data": "synthetic (seeded N(0,1))",
            "config": wl.config, "clocks": clock_info,
            "e2e": {"value": round(world * wl.value_work / (e2e_ms * 1e-3) / wl.value_scale, 3), "unit": wl.unit,
                    "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": sum(h.numel() * h.element_size() for h in host),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "gpu_launches": wl.launches * args.steps,
            "roofline": {"bound": wl.roof_bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                         "frac": round(achieved / peak, 4), "peak_source": peaks["source"],
                         "kernel_ms": round(kernel_ms, 4), "traffic": None,
                         **({"component_ms": components} if components else {}),
                         **({"component_frac_of_hbm": {
                             name: round(nbytes / (components[name] * 1e-3) / 1e9 / peaks["hbm"], 4)
                             for name, nbytes in kernel.component_bytes.items()}}
                            if hasattr(kernel, "component_bytes") else {})},
        }
        if not args.no_cpu_baseline and world == 1:
            torch.set_num_threads(os.cpu_count() or 1)
            sec, sample = wl.cpu_call()
            line["cpu_baseline"] = {"value": round(wl.value_work / sec / wl.value_scale, 5), "unit": wl.unit,
                                    "cores": torch.get_num_threads(), "kind": "port", "sample": sample,
                                    "ms_per_call_extrapolated": round(sec * 1e3, 2)}
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_workload_reference(args, wl) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        wl.cpu_call()
    samples = []
    for _ in range(args.steps):
        sec, sample = wl.cpu_call()
        samples.append(sec)
    sec = statistics.median(samples)
    value = wl.value_work / sec / wl.value_scale
    print(json.dumps({
        "impl": "reference", "metric": wl.metric, "value": round(value, 5), "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if wl.flush else "bf16", "data": "synthetic",
        "config": wl.config,
        "cpu_baseline": {"value": round(value, 5), "unit": wl.unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", default="b200", choices=["b200", "reference"])
    parser.add_argument("--heads-per-stage", type=int, default=4,
                        help="heads per copy/compute stage of the end-to-end (host memory) call")
    parser.add_argument("--workload", default="anima", choices=["anima", *WORKLOADS],
                        help="anima = the headline config 3; the others time the remaining configs")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--profile-only", action="store_true",
                        help="run warm-ups and K plain steps only (for ncu launch lists / captures)")
    parser.add_argument("--traffic", type=float, default=None,
                        help="dram bytes per attention launch from an ncu capture (reported as roofline.traffic)")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload != "anima":
        wl = WORKLOADS[args.workload]()
        (run_workload_reference if args.impl == "reference" else run_workload)(args, wl)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
