"""Benchmark of the MxWave hot path on B200 (one JSON line on rank 0).

Workload (one step): gamma-weighted MXFP4 quantization of an MLP up/gate
pair -- per-channel second moments of 8192 x 5120 bf16 calibration
activations (heavy-channel law) -> rms -> quantize two 17408 x 5120 bf16
weights (N(0, 0.015^2)) with the rms-weighted block error, percentile 99.5,
clip depth 1 (the reference defaults).  Inputs are synthetic (no checkpoint
offline) and larger than L2 (356 MB of weights per step).

``value`` is the whole-job rate of bf16 weight bytes quantized (GB/s) with
inputs resident in HBM; ``e2e`` is the same rate through the public Python
API from pinned host memory (H2D of weights + activations, D2H of packed
bytes and scales inside the timed region).  With --gpus N (torchrun) every
rank quantizes its own weights (row/tensor sharding, no communication) and
the time is the max over ranks.

``--impl reference`` times the CPU restatement of the reference's algorithm
(oracle port, all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TOKENS, HIDDEN, INTER = 8192, 5120, 17408
XTX_TOKENS = 65536
N_WEIGHTS = 2
DEPTH = 1
PCT = 99.5
BYTES_PER_ELEM = 2 + 0.5 + 1.0 / 32  # bf16 in, nibbles + E8M0 out
WORKLOAD = (
    f"gamma-weighted MXFP4 quantize of MLP up/gate {N_WEIGHTS}x{INTER}x{HIDDEN} bf16 "
    f"(rms from {TOKENS}x{HIDDEN} bf16 activations), pct {PCT}, depth {DEPTH}"
)
METRIC = "bf16 weight GB/s quantized"
# dram__bytes_read.sum + dram__bytes_write.sum of one quantize launch of this
# workload, from the ncu capture summarised in
# profiles/quantize_tma_kernel_gamma_d1_17408x5120.txt (178.37 MB + 26.45 MB).
QUANT_TRAFFIC_BYTES = 178_365_184 + 26_449_920
# The same for one X^T X launch (profiles/xtx_kernel_full_gram_65536x5120.txt).
XTX_TRAFFIC_BYTES = 1_682_721_000 + 92_257_536


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def _peaks_tensor() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured dense bf16 (burst)"
        except (KeyError, ValueError):
            pass
    return 1590.0, "fallback dense bf16"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self) -> dict:
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(smax), "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ our arm


def _bind_host_to_gpu(dev) -> dict:
    """Restrict this process's host threads to the CPUs NVML reports as local
    to its GPU, so that pinned staging buffers are first touched, and the copy
    threads run, on that GPU's NUMA node.  Read-only NVML queries; no GPU
    setting changes."""
    import torch

    try:
        import pynvml
    except ImportError:
        return {"bound": False, "why": "pynvml not importable"}
    props = torch.cuda.get_device_properties(dev)
    bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    try:
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            n = os.cpu_count() or 1
            mask = pynvml.nvmlDeviceGetCpuAffinity(handle, (n + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        return {"bound": False, "why": f"NVML: {exc}"}
    cpus = {64 * i + bit for i, word in enumerate(mask) for bit in range(64) if (int(word) >> bit) & 1}
    cpus &= os.sched_getaffinity(0)
    if not cpus:
        return {"bound": False, "why": "no local CPU in this process's affinity"}
    os.sched_setaffinity(0, cpus)
    return {"bound": True, "cpus": len(cpus), "pci": bus}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from mxwave_b200 import _lib, synthetic
    from mxwave_b200.core import quantize_mxfp4

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    host_binding = _bind_host_to_gpu(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    lib = _lib.load()

    x = synthetic.torch_activations(TOKENS, HIDDEN, seed=2 + 1000 * rank, device=dev)
    ws = [synthetic.torch_dense_weight(INTER, HIDDEN, seed=20 + i + 1000 * rank, device=dev, sigma=0.015,
                                       outlier_fraction=0.0) for i in range(N_WEIGHTS)]
    sum_sq = torch.zeros(HIDDEN, device=dev)
    rms = torch.empty(HIDDEN, device=dev)
    stream = torch.cuda.current_stream(dev)
    elems = N_WEIGHTS * INTER * HIDDEN
    ev_q = []

    def step(record: bool) -> list:
        cur = torch.cuda.current_stream(dev)  # the capture stream while a graph is recorded
        sum_sq.zero_()
        _lib.check(lib.mxw_accumulate_moments(x.data_ptr(), _lib.MXW_BF16, TOKENS, HIDDEN, HIDDEN, None,
                                              sum_sq.data_ptr(), cur.cuda_stream), "moments")
        _lib.check(lib.mxw_finalize_moments(None, sum_sq.data_ptr(), HIDDEN, TOKENS, None, rms.data_ptr(),
                                            cur.cuda_stream), "finalize")
        outs = []
        for w in ws:
            if record:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(cur)
            outs.append(quantize_mxfp4(w, scale_percentile=PCT, gamma=rms, mse_clip_depth=DEPTH))
            if record:
                b.record(cur)
                ev_q.append((a, b))
        return outs

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize(dev)
    # Per-launch duration of the quantize kernel (events around each launch).
    for _ in range(max(3, args.steps // 2)):
        step(True)
    torch.cuda.synchronize(dev)
    q_ms = sum(a.elapsed_time(b) for a, b in ev_q) / len(ev_q)
    # The step as one CUDA graph: the same launches, without per-launch host
    # overhead between them (the small moments/finalize kernels would
    # otherwise wait on the Python side).
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(False)
        graph.replay()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(0.3)
        start.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(False)
        stop.record(stream)
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    del graph

    # ---- end to end through the public API, host pinned buffers.
    e2e = None if args.no_e2e else run_e2e(args, dev, world, rank)
    # ---- calibration: X^T X on the tensor cores (config 3's token set).
    xtx = None if args.no_xtx else run_xtx(args, dev, world, rank)
    # ---- kernel timings of every objective and depth (rank 0 of one GPU).
    sweep = run_sweep(args, dev) if (world == 1 and not args.no_sweep) else None
    # ---- the decoder-layer, whole-checkpoint and engine workloads.
    layer = run_decoder_layer(args, dev) if (world == 1 and not args.no_layers) else None
    ckpt = None if args.no_layers else run_checkpoint_sweep(args, dev, world, rank)
    engine = run_engine(args, dev) if (world == 1 and not args.no_layers) else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = _peaks()
    bytes_per_launch = INTER * HIDDEN * BYTES_PER_ELEM + HIDDEN * 4
    achieved = bytes_per_launch / (q_ms * 1e-3) / 1e9
    value = world * elems * 2 * args.steps / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (bf16 in, u8 out)",
        "data": "synthetic (seeded on-device normal weights, heavy-channel activations)",
        "config": {"workload": WORKLOAD, "elements_per_step_per_gpu": elems, "l2": "inputs > L2 (356 MB weights)",
                   "parallelism": f"tensor-sharded x{world}, no collective",
                   "launch": "one CUDA graph per step" if not args.no_graph else "eager launches"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} copy bandwidth",
                     "traffic": args.traffic, "traffic_unit": "bytes per launch (ncu)",
                     "kernel": "quantize_tma_kernel<bf16,gamma,top2>",
                     "bytes_per_launch": int(bytes_per_launch), "avg_launch_ms": round(q_ms, 4)},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "calibration_xtx": xtx,
        "quantize_sweep": sweep,
        "decoder_layer": layer,
        "checkpoint_sweep": ckpt,
        "engine": engine,
        "gpu_launches": 6 * args.steps,  # moments, finalize, 2 x (quantize + rare-block fixup)
        "clocks": clocks.summary(),
        "host_binding": host_binding,
    }
    print(json.dumps(line), flush=True)


def run_e2e(args, dev, world: int, rank: int) -> dict:
    """Same step through the public API from pinned host memory to pinned host memory.

    ActivationCollector (moments kernel) on the host activations, then the
    ChunkStreamer (H2D / quantize / D2H overlapped on three streams) for both
    weights; the timed region holds every host<->device copy of the step.
    """
    import torch

    from mxwave_b200 import synthetic
    from mxwave_b200.calibration import ActivationCollector
    from mxwave_b200.streamer import ChunkStreamer

    x_h = synthetic.torch_activations(TOKENS, HIDDEN, seed=7 + rank, device=dev).cpu().pin_memory()
    w_h = [synthetic.torch_dense_weight(INTER, HIDDEN, seed=70 + i + rank, device=dev, sigma=0.015,
                                        outlier_fraction=0.0).cpu().pin_memory() for i in range(N_WEIGHTS)]
    p_h = [torch.empty((INTER, HIDDEN // 2), dtype=torch.uint8).pin_memory() for _ in range(N_WEIGHTS)]
    s_h = [torch.empty((INTER, HIDDEN // 32), dtype=torch.uint8).pin_memory() for _ in range(N_WEIGHTS)]
    streamer = ChunkStreamer(dev)
    stream = torch.cuda.current_stream(dev)

    def step() -> None:
        col = ActivationCollector({"mlp.weight": HIDDEN}, ("rms",))
        col.update("mlp.weight", x_h.to(dev, non_blocking=True))
        rms = col.finalize_on_device()["rms"]["mlp.weight"]
        for i, w in enumerate(w_h):
            streamer.quantize(w, p_h[i], s_h[i], scale_percentile=PCT, gamma=rms, mse_clip_depth=DEPTH)
        streamer.finish()

    for _ in range(max(2, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(2, args.steps // 2)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    elems = N_WEIGHTS * INTER * HIDDEN
    return {
        "value": round(world * elems * 2 * steps / (ms * 1e-3) / 1e9, 3),
        "unit": "GB/s",
        "h2d_bytes_per_step": int(elems * 2 + TOKENS * HIDDEN * 2),
        "d2h_bytes_per_step": int(elems // 2 + elems // 32),
        "ms_per_step": round(ms / steps, 3),
        "path": "ActivationCollector + ChunkStreamer (pinned host in/out, H2D/compute/D2H streams)",
    }


def run_xtx(args, dev, world: int, rank: int) -> dict:
    """Calibration X^T X: 65536 x 5120 bf16 tokens -> full fp32 Gram on tcgen05.

    Tokens are split across ranks (strong scaling); each rank accumulates its
    slice as packed upper-triangle tiles, one NCCL all-reduce sums those
    (55 MB against the full Gram's 105 MB), and each rank unpacks the sum.  Reported: whole-job
    tokens/s (max over ranks), and the tensor roofline of the local kernel.
    """
    import torch

    from mxwave_b200 import _lib, synthetic

    lib = _lib.load()
    total_tokens, k = XTX_TOKENS, HIDDEN
    lo, hi = total_tokens * rank // world, total_tokens * (rank + 1) // world
    x = synthetic.torch_activations(hi - lo, k, seed=300 + rank, device=dev)
    gram = torch.zeros(k, k, device=dev)
    stream = torch.cuda.current_stream(dev)

    # Several GPUs: each rank accumulates the packed upper-triangle tiles (55 MB
    # at 5120 channels instead of the full 105 MB Gram); one NCCL
    # reduce-scatter sums them and leaves each rank a band of whole tiles,
    # which it unpacks into its Gram: the summed Gram is distributed over the
    # ranks, band by band.
    tile_floats = 128 * 256
    n_tiles = int(lib.mxw_xtx_packed_tiles(k))
    per_rank = -(-n_tiles // world)
    packed = torch.zeros(per_rank * world * tile_floats, device=dev) if world > 1 else None
    band = torch.empty(per_rank * tile_floats, device=dev) if world > 1 else None

    def step(record=None) -> None:
        if world > 1:
            packed.zero_()
        else:
            gram.zero_()
        if record is not None:
            record[0].record(stream)
        if world > 1:
            _lib.check(lib.mxw_accumulate_xtx_packed(x.data_ptr(), hi - lo, k, k, packed.data_ptr(), None,
                                                     stream.cuda_stream), "xtx")
        else:
            _lib.check(lib.mxw_accumulate_xtx(x.data_ptr(), hi - lo, k, k, gram.data_ptr(), k, None,
                                              stream.cuda_stream), "xtx")
        if record is not None:
            record[1].record(stream)
        if world > 1:
            import torch.distributed as dist

            dist.reduce_scatter_tensor(band, packed, op=dist.ReduceOp.SUM)
            _lib.check(lib.mxw_xtx_unpack_tiles(band.data_ptr(), rank * per_rank, per_rank, k, gram.data_ptr(), k,
                                                stream.cuda_stream), "unpack")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(args.steps):
        step(kev[i])
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b)
    k_ms = sum(e0.elapsed_time(e1) for e0, e1 in kev) / len(kev)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms, k_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, k_ms = float(t[0]), float(t[1])
    peak = _peaks_tensor()
    # The Gram is symmetric: its k(k+1)/2 distinct entries take 2 flops per
    # token each.  The kernel runs the 128 x 256 tiles that reach the upper
    # triangle (row tile by holds column tiles by/2 ..); mma_flops counts them.
    n = hi - lo
    flops = 1.0 * n * k * (k + 1)
    tiles = sum((k + 255) // 256 - (by >> 1) for by in range(k // 128))
    mma_flops = 2.0 * n * 128 * 256 * tiles
    achieved = flops / (k_ms * 1e-3) / 1e12
    blocks = run_block_hessian(args, dev, world, rank, x, total_tokens, k)
    return {
        "metric": "calib tokens/s for X^T X",
        "block_hessian": blocks,
        "value": round(total_tokens * args.steps / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "scaling": "strong",
        "config": {"workload": f"full (symmetric) X^T X of {total_tokens} x {k} bf16 activations -> fp32 Gram, "
                               f"tokens split over {world} GPU(s)"
                               + (", NCCL reduce-scatter of the packed upper-triangle tiles, each rank unpacking "
                                  "its band (the summed Gram distributed by tile bands)" if world > 1 else "")},
        "ms_per_step": round(ms / args.steps, 4),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak[0], "unit": "TFLOP/s",
                     "frac": round(achieved / peak[0], 4), "peak_kind": peak[1], "kernel": "xtx_kernel (tcgen05)",
                     "traffic": XTX_TRAFFIC_BYTES if world == 1 else None, "traffic_unit": "bytes per launch (ncu)",
                     "flops_per_launch": flops, "mma_flops_per_launch": mma_flops,
                     "mma_tflops": round(mma_flops / (k_ms * 1e-3) / 1e12, 1), "avg_launch_ms": round(k_ms, 4)},
        "gpu_launches": args.steps,
    }


def run_block_hessian(args, dev, world: int, rank: int, x, total_tokens: int, k: int) -> dict:
    """The statistic the quantizer consumes: diagonal 32x32 blocks of X^T X.

    Each rank accumulates its token slice with the tensor-core block-Gram
    kernel, one NCCL all-reduce sums the [k/32, 32, 32] fp32 blocks
    (655 KB at 5120 channels), and every rank finalizes the damped block
    Hessian.  Whole-job tokens/s, max over ranks.
    """
    import torch

    from mxwave_b200 import _lib

    lib = _lib.load()
    n = x.shape[0]
    blocks = torch.zeros(k // 32, 32, 32, device=dev)
    hess = torch.empty_like(blocks)
    stream = torch.cuda.current_stream(dev)

    def step() -> None:
        blocks.zero_()
        _lib.check(lib.mxw_accumulate_block_gram(x.data_ptr(), _lib.MXW_BF16, n, k, k, blocks.data_ptr(),
                                                 stream.cuda_stream), "block gram")
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(blocks, op=dist.ReduceOp.SUM)
        _lib.check(lib.mxw_finalize_block_hessian(blocks.data_ptr(), 0, k, k, total_tokens, 1e-6,
                                                  _lib.MXW_DAMP_ABSOLUTE, hess.data_ptr(), stream.cuda_stream),
                   "finalize")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    peak, _kind = _peaks()
    return {
        "workload": f"diagonal 32x32 blocks of X^T X of {total_tokens} x {k} bf16 tokens (tensor cores), "
                    f"tokens split over {world} GPU(s)" + (", NCCL all-reduce of the blocks" if world > 1 else ""),
        "value": round(total_tokens * args.steps / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "ms_per_step": round(ms / args.steps, 4),
        "hbm_frac_per_gpu": round(n * k * 2 / (ms / args.steps * 1e-3) / 1e9 / peak, 4),
    }


def _flush_l2(buf) -> None:
    buf.zero_()


def _time_launches(fn, flush, reps: int) -> float:
    """Median device time (ms) of fn() over reps launches, L2 flushed before each."""
    import torch

    times = []
    for _ in range(reps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def run_sweep(args, dev) -> dict:
    """Quantize kernel timings per objective and depth on one 17408 x 5120 bf16 weight.

    Every setting of the reference's quantize_mxfp4 that the workloads use:
    unweighted (depth 1 and 4, percentile 100), gamma-weighted (depth 1, 4),
    rtn, and the block-Hessian objective (depth 1, 4) with the 32x32 blocks of
    the X^T X of 65536 heavy-channel tokens (damp 1e-6, absolute).  Each
    number is the median of CUDA-event times around single launches (main
    pass + rare-block pass) with L2 flushed before each; the roofline is the
    algorithmic bytes (2.53125 B per weight + gamma / Hessian bytes) over that
    time against the measured HBM copy bandwidth.
    """
    import torch

    from mxwave_b200 import _lib, synthetic
    from mxwave_b200.core import quantize_into

    lib = _lib.load()
    peak, peak_kind = _peaks()
    w = synthetic.torch_dense_weight(INTER, HIDDEN, seed=31, device=dev, sigma=0.015)
    x = synthetic.torch_activations(XTX_TOKENS, HIDDEN, seed=300, device=dev)
    gram = torch.zeros(HIDDEN, HIDDEN, device=dev)
    _lib.check(lib.mxw_accumulate_xtx(x.data_ptr(), XTX_TOKENS, HIDDEN, HIDDEN, gram.data_ptr(), HIDDEN, None,
                                      torch.cuda.current_stream(dev).cuda_stream), "xtx")
    hess = torch.empty(HIDDEN // 32, 32, 32, device=dev)
    _lib.check(lib.mxw_finalize_block_hessian(gram.data_ptr(), 1, HIDDEN, HIDDEN, XTX_TOKENS, 1e-6,
                                              _lib.MXW_DAMP_ABSOLUTE, hess.data_ptr(),
                                              torch.cuda.current_stream(dev).cuda_stream), "finalize")
    del x, gram
    xs = synthetic.torch_activations(TOKENS, HIDDEN, seed=2, device=dev).float()
    gamma = xs.square().mean(0).sqrt()
    del xs
    pk = torch.empty(INTER, HIDDEN // 2, dtype=torch.uint8, device=dev)
    sc = torch.empty(INTER, HIDDEN // 32, dtype=torch.uint8, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    settings = [
        ("unweighted_d1", {}, 0), ("unweighted_d4", {"mse_clip_depth": 4}, 0),
        ("unweighted_pct100_d1", {"scale_percentile": 100.0}, 0),
        ("gamma_d1", {"gamma": gamma}, HIDDEN * 4), ("gamma_d4", {"gamma": gamma, "mse_clip_depth": 4}, HIDDEN * 4),
        ("rtn", {"method": "rtn"}, 0),
        ("hessian_d1", {"hessian": hess}, HIDDEN * 128), ("hessian_d4", {"hessian": hess, "mse_clip_depth": 4},
                                                          HIDDEN * 128),
    ]
    out = {}
    for name, kw, extra in settings:
        def launch(kw=kw) -> None:
            flags.zero_()
            quantize_into(w, pk, sc, flags=flags, **kw)

        for _ in range(3):
            launch()
        ms = _time_launches(launch, lambda: _flush_l2(flush), 9)
        nbytes = INTER * HIDDEN * BYTES_PER_ELEM + extra
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 1), "algorithmic_GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
                     "bf16_weight_GBps": round(INTER * HIDDEN * 2 / (ms * 1e-3) / 1e9, 1)}
    del pk, sc, w, flush
    return {"workload": f"one {INTER} x {HIDDEN} bf16 weight per setting, pct {PCT} unless stated; Hessian blocks "
                        f"from the X^T X of {XTX_TOKENS} heavy-channel tokens",
            "peak_GBps": peak, "peak_kind": f"{peak_kind} copy bandwidth", "l2": "flushed before every launch",
            "timing": "median of 9 single launches (main + rare-block pass), CUDA events", "settings": out,
            "dense4096_graph64": _dense4096_graph(dev, peak)}


def _dense4096_graph(dev, peak: float) -> dict:
    """The dense 4096 x 4096 workload as 64 distinct weights quantized in one CUDA graph.

    N(0, 0.02^2) with 0.1 % outliers x20 (the same law as the golden 4096^2
    case), unweighted depth 1 and 4 and rtn; 2.1 GB of weights per replay, so
    every launch reads from HBM.  Median of 5 replays.
    """
    import torch

    from mxwave_b200 import synthetic
    from mxwave_b200.core import quantize_into

    n, k = 64, 4096
    ws = [synthetic.torch_dense_weight(k, k, seed=700 + i, device=dev) for i in range(n)]
    pk = torch.empty(k, k // 2, dtype=torch.uint8, device=dev)
    sc = torch.empty(k, k // 32, dtype=torch.uint8, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    out = {}
    for name, kw in (("mse_d1", {}), ("mse_d4", {"mse_clip_depth": 4}), ("rtn", {"method": "rtn"})):
        def batch(kw=kw) -> None:
            for w in ws:
                quantize_into(w, pk, sc, flags=flags, **kw)

        batch()
        torch.cuda.synchronize(dev)
        side = torch.cuda.Stream(dev)
        with torch.cuda.stream(side):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                batch()
        torch.cuda.synchronize(dev)
        graph.replay()
        times = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b))
        del graph
        ms = sorted(times)[2]
        nbytes = n * k * k * BYTES_PER_ELEM
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us_per_tensor": round(ms * 1e3 / n, 1), "algorithmic_GBps": round(gbs, 1),
                     "frac": round(gbs / peak, 4), "bf16_weight_GBps": round(n * k * k * 2 / (ms * 1e-3) / 1e9, 1)}
    del ws
    return {"workload": f"{n} distinct {k} x {k} bf16 weights per CUDA graph replay", **out}


LAYER_LINEARS = (("self_attn.q_proj", 5120), ("self_attn.k_proj", 5120), ("self_attn.v_proj", 5120),
                 ("self_attn.o_proj", 5120), ("mlp.gate_proj", 5120), ("mlp.up_proj", 5120),
                 ("mlp.down_proj", 17408))


def run_decoder_layer(args, dev) -> dict:
    """Decoder-layer workload: layer-streamed calibration, then all seven linears quantized.

    A random-init Qwen3.5 decoder layer (hidden 5120, gated q_proj, GQA 40/8 of
    128, SwiGLU 17408, vocabulary 151936) in a safetensors checkpoint; 128
    sequences x 2048 uniformly random token ids.  Calibration is
    mxwave_b200.calibration_stream.calibrate_decoder_sequentially (bf16, rms +
    block-Hessian statistics of every linear input, hidden states kept in
    HBM), timed wall-clock from checkpoint to finalized statistics.  Then the
    seven linears are quantized from HBM with their block Hessians and, as a
    second pass, their rms gammas (depth 1), timed with CUDA events.
    """
    import tempfile

    import torch
    from safetensors import safe_open

    from mxwave_b200 import synthetic
    from mxwave_b200.calibration_stream import calibrate_decoder_sequentially
    from mxwave_b200.core import quantize_into

    _reference_importable()
    cfg = synthetic.decoder_config(layers=1)
    seqs, length = 128, 2048
    g = torch.Generator().manual_seed(44)
    ids = torch.randint(0, cfg.vocab_size, (seqs, length), generator=g).tolist()
    targets = {f"model.layers.0.{n}.weight": w for n, w in LAYER_LINEARS}
    objectives = ("rms", "block-hessian")
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "model.safetensors"
        files = synthetic.write_decoder_checkpoint(path, cfg, seed=4000, device=dev)
        kw = dict(device=dev, dtype=torch.bfloat16, batch_size=16, hessian_damp=1e-6)
        calibrate_decoder_sequentially(synthetic.meta_decoder(cfg), targets, objectives, ids[:16], files, **kw)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        res = calibrate_decoder_sequentially(synthetic.meta_decoder(cfg), targets, objectives, ids, files, **kw)
        torch.cuda.synchronize(dev)
        cal_s = time.perf_counter() - t0
        with safe_open(str(path), framework="pt", device=str(dev)) as f:
            weights = {n: f.get_tensor(n) for n in targets}
    peak, peak_kind = _peaks()
    out = {}
    elems = sum(w.numel() for w in weights.values())
    for objective, key in (("block-hessian", "hessian"), ("rms", "gamma")):
        stats = {n: res.statistics[objective][n].to(dev) for n in targets}
        bufs = {n: (torch.empty(w.shape[0], w.shape[1] // 2, dtype=torch.uint8, device=dev),
                    torch.empty(w.shape[0], w.shape[1] // 32, dtype=torch.uint8, device=dev))
                for n, w in weights.items()}

        def launch() -> None:
            for n, w in weights.items():
                quantize_into(w, bufs[n][0], bufs[n][1], mse_clip_depth=1, **{key: stats[n]})

        launch()
        reps = 5
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            launch()
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b) / reps
        nbytes = elems * BYTES_PER_ELEM + sum(s.numel() * 4 for s in stats.values())
        out[f"{objective}_d1"] = {"ms_per_layer": round(ms, 3),
                                  "bf16_weight_GBps": round(elems * 2 / (ms * 1e-3) / 1e9, 1),
                                  "roofline_frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)}
    tokens = seqs * length
    return {
        "workload": "random-init Qwen3.5 decoder layer (hidden 5120, GQA 40/8 x 128, gated q, SwiGLU 17408, "
                    "vocab 151936), 128 x 2048 random token ids; rms + block-Hessian statistics of all 7 linear "
                    "inputs, then all 7 linears quantized (depth 1)",
        "calibration": {"tokens": tokens, "seconds": round(cal_s, 3), "tokens_per_s": round(tokens / cal_s, 1),
                        "timing": "wall clock, checkpoint to finalized statistics, one layer"},
        "quantize": out,
        "weight_elements_per_layer": elems,
        "peak_kind": f"{peak_kind} copy bandwidth",
    }


def _reference_importable() -> None:
    ref = ROOT / "baseline" / "_ref"
    if (ref / "mxwave").exists() and str(ref) not in sys.path:
        sys.path.insert(0, str(ref))


def _h2d_bandwidth(dev) -> float:
    """Pinned host -> device copy bandwidth (GB/s) of one 1 GiB copy, best of 3."""
    import torch

    src = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, (1 << 30) / (a.elapsed_time(b) * 1e-3) / 1e9)
    return best


def run_checkpoint_sweep(args, dev, world: int, rank: int) -> dict:
    """Whole-checkpoint workload (a stated subset): host-pinned layers + the MoE expert stack.

    4 decoder layers of the decoder-layer shape (7 linears each) and 128 routed
    experts (gate/up 768 x 2048, down 2048 x 768) live in pinned host memory
    and stream through ChunkStreamer (H2D / quantize / D2H on three streams)
    with block-Hessian weighting at depth 1 (one synthetic Hessian per input
    width).  Tensors are dealt round-robin over the ranks.  Reported: the
    whole-job bf16 weight rate, its fraction of the measured pinned H2D link
    bandwidth, and the kernel-only HBM fraction (the same quantize launches
    with the weights resident in HBM).
    """
    import torch

    from mxwave_b200 import synthetic
    from mxwave_b200.core import compute_block_hessian, quantize_into
    from mxwave_b200.streamer import ChunkStreamer

    layers, experts = 4, 128
    shapes = []
    for layer in range(layers):
        for n, k in LAYER_LINEARS:
            rows = {"self_attn.q_proj": 10240, "self_attn.k_proj": 1024, "self_attn.v_proj": 1024,
                    "self_attn.o_proj": 5120, "mlp.gate_proj": 17408, "mlp.up_proj": 17408,
                    "mlp.down_proj": 5120}[n]
            shapes.append((rows, k))
    for _ in range(experts):
        shapes += [(768, 2048), (768, 2048), (2048, 768)]
    mine = [(i, s) for i, s in enumerate(shapes) if i % world == rank]
    hess = {k: compute_block_hessian(synthetic.torch_activations(8192, k, seed=600 + k, device=dev))
            for k in sorted({k for _, k in shapes})}
    host = []
    for i, (r, k) in mine:
        w = synthetic.torch_dense_weight(r, k, seed=9000 + i, device=dev, outlier_fraction=0.0)
        host.append((w.cpu().pin_memory(), k))
    outs = [(torch.empty(w.shape[0], w.shape[1] // 2, dtype=torch.uint8).pin_memory(),
             torch.empty(w.shape[0], w.shape[1] // 32, dtype=torch.uint8).pin_memory()) for w, _ in host]
    link = _h2d_bandwidth(dev)
    streamer = ChunkStreamer(dev)

    def sweep() -> None:
        for (w, k), (p, s) in zip(host, outs):
            streamer.quantize(w, p, s, hessian=hess[k], mse_clip_depth=1)
        streamer.finish()

    sweep()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    sweep()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b)
    # Kernel-only: the same launches with every weight resident in HBM,
    # captured once in a CUDA graph and replayed, so that host launch overhead
    # (large beside the 768 x 2048 expert kernels) stays out of the figure.
    dev_w = [(w.to(dev), k) for w, k in host]
    dev_o = [(torch.empty(w.shape[0], w.shape[1] // 2, dtype=torch.uint8, device=dev),
              torch.empty(w.shape[0], w.shape[1] // 32, dtype=torch.uint8, device=dev)) for w, _ in dev_w]

    def resident() -> None:
        for (wd, k), (pk, sc) in zip(dev_w, dev_o):
            quantize_into(wd, pk, sc, hessian=hess[k], mse_clip_depth=1)

    resident()
    torch.cuda.synchronize(dev)
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            resident()
    torch.cuda.synchronize(dev)
    graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    e1.synchronize()
    k_ms = e0.elapsed_time(e1)
    del graph, dev_w, dev_o
    elems_local = sum(w.numel() for w, _ in host)
    elems_total = sum(r * k for r, k in shapes)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms, k_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, k_ms = float(t[0]), float(t[1])
    peak, peak_kind = _peaks()
    h2d_rate = elems_local * 2 / (ms * 1e-3) / 1e9
    return {
        "workload": f"{layers} decoder layers (7 linears of the decoder-layer shape) + {experts} experts "
                    "(gate/up 768x2048, down 2048x768) bf16 in pinned host memory, block-Hessian depth 1, "
                    f"tensors round-robin over {world} GPU(s)",
        "subset": "4 of the 64 layers and one MoE layer of the whole-checkpoint workload",
        "value": round(elems_total * 2 / (ms * 1e-3) / 1e9, 2),
        "unit": "GB/s bf16 weight (whole job)",
        "ms": round(ms, 2),
        "weight_elements": elems_total,
        "link": {"h2d_GBps_measured": round(link, 1), "h2d_GBps_achieved_per_gpu": round(h2d_rate, 1),
                 "frac": round(h2d_rate / link, 4),
                 "bytes_per_gpu": int(elems_local * 2 + elems_local * (0.5 + 1 / 32))},
        "kernel_only": {"ms_per_gpu": round(k_ms, 2), "timing": "one CUDA graph of every quantize launch, weights resident",
                        "hbm_frac": round(elems_local * BYTES_PER_ELEM / (k_ms * 1e-3) / 1e9 / peak, 4),
                        "peak_kind": f"{peak_kind} copy bandwidth"},
    }


def run_engine(args, dev) -> dict:
    """mxwave.engine.quantize_model on a synthetic two-shard checkpoint, with and without this package.

    The checkpoint holds two decoder layers of the decoder-layer shape (seven
    linears each, bf16) plus their norms.  The reference engine runs on the
    GPU twice: with its own torch implementation of the hot path, and with
    this package installed (quantizer, chunk stream, SQNR off).  Wall clock of
    quantize_model (planning, shard writing and fsync included).  The output
    shards of the two runs are compared byte for byte and reported; parity is
    defined against the reference's CPU path (which this package reproduces
    bit for bit), and its torch GPU path is not guaranteed to equal that.
    """
    import hashlib
    import tempfile

    import torch
    from safetensors.torch import save_file

    from mxwave_b200 import synthetic

    _reference_importable()
    try:
        import mxwave.engine as engine
    except ImportError:
        return {"unavailable": "reference package not installed in baseline/_ref"}
    from mxwave_b200.install import install

    shapes = {"self_attn.q_proj": (10240, 5120), "self_attn.k_proj": (1024, 5120), "self_attn.v_proj": (1024, 5120),
              "self_attn.o_proj": (5120, 5120), "mlp.gate_proj": (17408, 5120), "mlp.up_proj": (17408, 5120),
              "mlp.down_proj": (5120, 17408)}
    with tempfile.TemporaryDirectory() as tmp:
        model = Path(tmp) / "model"
        model.mkdir()
        weight_map = {}
        elems = 0
        for layer in range(2):
            shard = {}
            for i, (n, (r, k)) in enumerate(shapes.items()):
                name = f"model.layers.{layer}.{n}.weight"
                shard[name] = synthetic.torch_dense_weight(r, k, seed=5000 + 10 * layer + i, device=dev).cpu()
                elems += r * k
            shard[f"model.layers.{layer}.input_layernorm.weight"] = torch.ones(5120, dtype=torch.bfloat16)
            fname = f"model-{layer + 1:05d}-of-00002.safetensors"
            save_file(shard, str(model / fname))
            weight_map.update({k: fname for k in shard})
        (model / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
        (model / "config.json").write_text(json.dumps({"model_type": "test"}))
        (model / "tokenizer.json").write_text('{"version":"1.0"}')
        common = dict(model_dir=model, policy="all-linear", verbose=False, device=str(dev))

        def run(out: Path) -> float:
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            engine_mod = sys.modules["mxwave.engine"]
            engine_mod.quantize_model(engine_mod.QuantizeConfig(output_dir=out, **common))
            torch.cuda.synchronize(dev)
            return time.perf_counter() - t0

        def digest(out: Path) -> str:
            h = hashlib.sha256()
            for f in sorted(out.glob("*.safetensors")):
                h.update(f.read_bytes())
            return h.hexdigest()

        ref_s = run(Path(tmp) / "ref")
        handle = install()
        try:
            run(Path(tmp) / "warm")
            ours_s = run(Path(tmp) / "ours")
        finally:
            handle.uninstall()
        same = digest(Path(tmp) / "ref") == digest(Path(tmp) / "ours")
    gb = elems * 2 / 1e9
    return {
        "workload": "mxwave.engine.quantize_model, 2 shards x 7 linears of the decoder-layer shape (bf16), "
                    "policy all-linear, mse depth 1, one GPU",
        "ours": {"seconds": round(ours_s, 3), "bf16_weight_GBps": round(gb / ours_s, 2)},
        "reference_on_gpu": {"seconds": round(ref_s, 3), "bf16_weight_GBps": round(gb / ref_s, 2),
                             "path": "the reference's own torch quantize_mxfp4 and chunk loop on the same GPU"},
        "speedup": round(ref_s / ours_s, 2),
        "identical_to_reference_gpu_run": same,
        "weight_elements": elems,
    }


# ---------------------------------------------------------- CPU reference


def _oracle_sample(rows: int):
    """A row sample of the workload for the CPU restatement (numpy inputs)."""
    import numpy as np

    from mxwave_b200 import synthetic

    x = synthetic.bf16_bits_to_f32(synthetic.det_activations(1024, HIDDEN, seed=2)).astype(np.float64)
    gamma = np.sqrt((x * x).mean(0)).astype(np.float32)
    ws = [synthetic.det_dense_weight(rows, HIDDEN, seed=20 + i, sigma=0.015, outlier_fraction=0.0)
          for i in range(N_WEIGHTS)]
    return ws, gamma


def cpu_baseline(seconds: float) -> dict:
    """Time the oracle port of the reference algorithm on the host cores."""
    from oracle import oracle

    threads = oracle.default_threads()
    ws, gamma = _oracle_sample(256)
    t0 = time.perf_counter()
    for w in ws:
        oracle.quantize_mxfp4(w, PCT, gamma=gamma, mse_clip_depth=DEPTH, threads=threads)
    probe = time.perf_counter() - t0
    rows = int(max(64, min(INTER, 256 * seconds / max(probe, 1e-3))))
    ws, gamma = _oracle_sample(rows)
    t0 = time.perf_counter()
    for w in ws:
        oracle.quantize_mxfp4(w, PCT, gamma=gamma, mse_clip_depth=DEPTH, threads=threads)
    dt = time.perf_counter() - t0
    elems = N_WEIGHTS * rows * HIDDEN
    return {"value": round(elems * 2 / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{N_WEIGHTS} x {rows} rows x {HIDDEN} of the workload's weights ({dt:.1f} s)"}


def _cpu_model() -> str | None:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def reference_python(seconds: float) -> dict:
    """The reference's own Python (baseline/_ref) on the host cores: a bounded row sample.

    mxwave.checkpoint.iter_quantized_row_chunks + mxwave.core.quantize_mxfp4
    on CPU fp32 with torch using every host thread, on rows of the workload's
    weights (gamma from the reference's own ActivationCollector).
    """
    import platform

    import numpy as np
    import torch

    _reference_importable()
    try:
        from mxwave import calibration as ref_cal
        from mxwave import checkpoint as ref_ckpt
        from mxwave import core as ref_core
    except ImportError:
        return {"unavailable": "reference package not installed in baseline/_ref"}
    from mxwave_b200 import synthetic

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    xb = synthetic.det_activations(1024, HIDDEN, seed=2)
    col = ref_cal.ActivationCollector({"mlp.weight": HIDDEN}, ("rms",))
    col.update("mlp.weight", torch.from_numpy(xb.view(np.int16).copy()).view(torch.bfloat16))
    gamma = col.finalize()["rms"]["mlp.weight"]

    def quantize(rows: int) -> float:
        bits = synthetic.det_dense_weight(rows, HIDDEN, seed=20, sigma=0.015, outlier_fraction=0.0)
        w = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
        t0 = time.perf_counter()
        for _ in ref_ckpt.iter_quantized_row_chunks(
                lambda a, b: w[a:b], lambda c: ref_core.quantize_mxfp4(c, PCT, gamma=gamma, mse_clip_depth=DEPTH),
                rows=rows, columns=HIDDEN, max_rows=1024, max_elements=ref_ckpt.DEFAULT_TENSOR_CHUNK_MAX_ELEMENTS,
                name="w"):
            pass
        return time.perf_counter() - t0

    probe = quantize(204)
    rows = int(max(204, min(INTER, 204 * seconds / max(probe, 1e-3))))
    dt = quantize(rows)
    return {"value": round(rows * HIDDEN * 2 / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "reference",
            "cpu": _cpu_model() or platform.machine(),
            "sample": f"{rows} rows x {HIDDEN} of one workload weight through the reference's chunk loop "
                      f"({dt:.1f} s)"}


def reference_python_workloads(seconds: float) -> dict:
    """The reference's own Python on the host cores for the other workloads, each a bounded sample.

    * dense 4096 x 4096 (unweighted, depth 1) through its chunk loop;
    * block-Hessian depth 4 on rows of a 17408 x 5120 weight, Hessian blocks from
      the reference collector on 1024 heavy-channel tokens;
    * calibration: ActivationCollector.update (rms + block Hessian) and the fp32
      X^T X (torch matmul, the product the reference does not form) on 4096 tokens.
    """
    import numpy as np
    import torch

    _reference_importable()
    try:
        from mxwave import calibration as ref_cal
        from mxwave import checkpoint as ref_ckpt
        from mxwave import core as ref_core
    except ImportError:
        return {"unavailable": "reference package not installed in baseline/_ref"}
    from mxwave_b200 import synthetic

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)

    def bf16(bits):
        return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)

    def chunked(w, cols, **kw) -> float:
        rows = w.shape[0]
        t0 = time.perf_counter()
        for _ in ref_ckpt.iter_quantized_row_chunks(
                lambda a, b: w[a:b], lambda c: ref_core.quantize_mxfp4(c, **kw), rows=rows, columns=cols,
                max_rows=1024, max_elements=ref_ckpt.DEFAULT_TENSOR_CHUNK_MAX_ELEMENTS, name="w"):
            pass
        return time.perf_counter() - t0

    def sampled(bits, cols, **kw) -> tuple[int, float]:
        w = bf16(bits)
        probe = chunked(w[:256], cols, **kw)
        rows = int(max(256, min(w.shape[0], 256 * seconds / max(probe, 1e-3))))
        return rows, chunked(w[:rows], cols, **kw)

    out = {"cores": threads, "kind": "reference"}
    rows, dt = sampled(synthetic.det_dense_weight(4096, 4096, seed=0), 4096)
    out["dense4096_mse_d1"] = {"value": round(rows * 4096 * 2 / dt / 1e9, 4), "unit": "GB/s",
                               "sample": f"{rows} of 4096 rows ({dt:.1f} s)"}
    xb = bf16(synthetic.det_activations(1024, HIDDEN, seed=300))
    col = ref_cal.ActivationCollector({"w.weight": HIDDEN}, ("block-hessian",))
    col.update("w.weight", xb)
    hess = col.finalize()["block-hessian"]["w.weight"]
    rows, dt = sampled(synthetic.det_dense_weight(INTER, HIDDEN, seed=31, sigma=0.015), HIDDEN, hessian=hess,
                       mse_clip_depth=4)
    out["hessian_d4"] = {"value": round(rows * HIDDEN * 2 / dt / 1e9, 4), "unit": "GB/s",
                         "sample": f"{rows} of {INTER} rows x {HIDDEN} ({dt:.1f} s)"}
    n = 4096
    xc = bf16(synthetic.det_activations(n, HIDDEN, seed=2))
    col = ref_cal.ActivationCollector({"w.weight": HIDDEN}, ("rms", "block-hessian"))
    t0 = time.perf_counter()
    col.update("w.weight", xc)
    dt_col = time.perf_counter() - t0
    xf = xc.float()
    t0 = time.perf_counter()
    _ = xf.T @ xf
    dt_xtx = time.perf_counter() - t0
    out["collector_update_tokens_per_s"] = round(n / dt_col, 1)
    out["xtx_fp32_tokens_per_s"] = round(n / dt_xtx, 1)
    out["calibration_sample"] = f"{n} x {HIDDEN} bf16 tokens"
    return out


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle

    threads = oracle.default_threads()
    # The full workload per step: both 17408 x 5120 weights (about 1.3 s on 16 threads).
    rows = INTER
    ws, gamma = _oracle_sample(rows)

    def step() -> None:
        for w in ws:
            oracle.quantize_mxfp4(w, PCT, gamma=gamma, mse_clip_depth=DEPTH, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    elems = N_WEIGHTS * rows * HIDDEN
    value = elems * 2 * args.steps / dt / 1e9
    sample = f"the whole workload: {N_WEIGHTS} x {rows} rows x {HIDDEN} per step"
    py = None if args.no_reference_python else reference_python(args.cpu_seconds)
    py_more = None if args.no_reference_python else reference_python_workloads(args.cpu_seconds / 3)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (bf16 in, u8 out)",
        "data": "synthetic (seeded, platform-independent generator)",
        "config": {"workload": WORKLOAD, "sample": sample},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "reference_python": py,
        "reference_python_workloads": py_more,
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-xtx", action="store_true", help="skip the X^T X calibration measurement")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--no-graph", action="store_true", help="launch the timed steps one kernel at a time")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-objective quantize kernel timings")
    ap.add_argument("--no-reference-python", action="store_true",
                    help="--impl reference: skip timing the reference's own Python beside the port")
    ap.add_argument("--no-layers", action="store_true",
                    help="skip the decoder-layer, whole-checkpoint and engine workloads")
    ap.add_argument("--traffic", type=float, default=QUANT_TRAFFIC_BYTES,
                    help="dram bytes per quantize launch from an ncu capture (recorded in the roofline)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
