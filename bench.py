"""Benchmark of the quantized linear stage (one JSON line on rank 0).

Default workload (config 1 of the benchmark configs, the one the headline metric is quoted on):
one int8 weight-only linear, x bf16 [4096, 3072], W int8 [3072, 3072] per-output-channel scales,
bf16 bias, fp32 accumulation, bf16 output.  A step is one product over that batch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg1|cfg2|gemv1|gemv4|gemv16|gemv32|prefill128|...]
  python bench.py --impl reference ...   # the reference's CPU path (the oracle), on the host cores

With N > 1 (one process per GPU under torch.distributed.run) config 1 runs column-parallel: rank r
multiplies x by its block of W's columns and the product's epilogue stores every output tile into every
rank's y over NVLink, so each rank ends the step holding the whole y (strong scaling; ``run_scale``,
with a bit-exact check against one GPU's product before timing).  ``--workload cfg1-replicas`` (and
the other workloads) give every rank its own batch with the weight replicated instead (batch sharding,
no collective on the data path); ``value`` is the work of all ranks over the slowest rank's time.
Timing: W untimed warm-up steps, then K timed steps, each bracketed by CUDA events on the launching
stream, with the L2 flushed (a 256 MiB write, then a 256 MiB read of another buffer so that the L2
holds clean lines) before every step; barrier + synchronize around the
timed region; the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_FLUSH_BYTES = 256 << 20


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))}, "measured"
    return dict(FALLBACK_PEAKS, bf16_tflops_sustained=1400.0), "fallback"


def make_case(workload: str):
    from siliconed_b200 import configs
    if workload in ("cfg1", "cfg1-w8a8", "cfg1-replicas"):
        return configs.config1()
    if workload == "cfg2":
        return configs.config2()
    if workload.startswith("gemv"):
        m = int(workload[4:] or 1)
        return configs.config4(m, 12288, 4096)
    if workload.startswith("prefill"):
        m = int(workload[7:] or 128)
        if not 32 < m <= 128:
            raise SystemExit("prefillM takes 32 < M <= 128")
        return configs.encoder_prefill(m)
    raise SystemExit(f"unknown workload {workload}")


def parallelism_of(workload: str, world: int) -> str:
    """How N > 1 GPUs share a step: config 1 (the default) splits W's columns over the ranks and gathers y
    inside the product (strong scaling); `cfg1-replicas` and the GEMV workloads give every rank a whole
    product (weak scaling)."""
    if world <= 1:
        return "one GPU"
    if workload == "cfg1":
        return f"column-parallel x{world}: W's columns split over the ranks, y gathered in the product's epilogue"
    return f"replicas x{world} (batch-sharded)"


def describe(case, workload, world=1):
    bound = "hbm" if case.m <= 32 else "tensor"
    return {"workload": f"{workload}: {case.name} x bf16 [{case.m}, {case.k}] . W [{case.k}, {case.n}] "
                        f"{'int8' if case.kind == 1 else 'e4m3'} per-channel, fp32 accumulate, bf16 out",
            "m": case.m, "k": case.k, "n": case.n, "bias": case.bias is not None, "bound": bound,
            "l2": "flushed before every timed step (256 MiB write, then a 256 MiB read that leaves the L2 clean)",
            "parallelism": parallelism_of(workload, world)}


def metric_of(case):
    if case.m <= 32:
        return "int8-weight GEMV achieved HBM GB/s", "GB/s"
    if case.m <= 128:
        return f"int8-weight GEMM TFLOP/s at M={case.m} (encoder prefill)", "TFLOP/s"
    return "int8-weight GEMM TFLOP/s at M=4096" if case.kind == 1 else "fp8-weight GEMM TFLOP/s at M=4096", "TFLOP/s"


def throughput(case, seconds, unit, ranks=1):
    if unit == "GB/s":
        return ranks * case.bytes_moved() / seconds / 1e9
    return ranks * case.flops / seconds / 1e12


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, v in enumerate(flags) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def route_kernels(case, ws_bytes: int) -> list[str]:
    """The library's kernels one product of this case launches (the step the roofline's `achieved`
    covers): the GEMV up to 4 rows (an int8 weight of 3-16 rows with the workspace: the integer skinny
    product), the skinny tensor-core product up to 32, the single-CTA GEMM up
    to 128 rows, the fused pair kernel above, and from 1536 rows with a workspace the widening of the
    codes followed by the bf16-operand pair GEMM."""
    if case.m <= 16 and case.m > 2 and case.kind == 1 and ws_bytes > 0:
        return ["x_planes", "gemm_i8_skinny"]
    if case.m <= 4:
        return ["gemv_w8"]
    if case.m <= 16 and case.kind == 1 and ws_bytes > 0:
        return ["x_planes", "gemm_i8_skinny"]
    if case.m <= 32:
        return ["gemm_w8_skinny"]
    if case.m <= 128:
        return ["gemm_w8_tc"]
    if ws_bytes > 0:
        # 2 to 3 rounds of 256 x 256 pair tiles in one group of the tile order: the widening runs inside
        # the GEMM (fused_widen_fits in the library)
        import torch
        pairs = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count // 2
        m_tiles, n_tiles = -(-case.m // 256), -(-case.n // 256)
        if m_tiles <= 16 and 2 * pairs <= m_tiles * n_tiles <= 3 * pairs:
            return ["gemm_bf16_pair (widening inside)"]
        return ["widen_codes", "gemm_bf16_pair"]
    return ["gemm_w8_pair"]


def cpu_baseline(case, budget_s: float = 12.0, steps: int | None = None, warmup: int = 0):
    """The reference's CPU path restated (the oracle): dequantize W (OpenMP, all host threads), then
    an fp32 GEMM on the CPU (torch.matmul, all threads), on a bounded sample of the rows.  Timed
    repetitions run until `budget_s` (at most 1000), or exactly `steps` after `warmup` untimed ones."""
    import torch
    import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    torch.set_num_threads(threads)
    codes_kn = np.ascontiguousarray(case.codes_nk.T)
    rows = case.m if case.m <= 32 else 256
    x = torch.from_numpy(((case.x[:rows].astype(np.uint32) << 16).view(np.float32)).copy())
    bias = None if case.bias is None else torch.from_numpy((case.bias.astype(np.uint32) << 16).view(np.float32))
    reps, t_total = 0, 0.0
    for i in range(-warmup, 10 ** 9):
        if steps is not None and reps >= steps:
            break
        if steps is None and reps > 0 and (t_total >= budget_s or reps >= 1000):
            break
        t0 = time.perf_counter()
        w = oracle.dequantize(codes_kn, case.kind, case.scales, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS,
                              case.n).reshape(case.k, case.n)
        y = x @ torch.from_numpy(w)
        if bias is not None:
            y += bias
        if i >= 0:
            t_total += time.perf_counter() - t0
            reps += 1
    per = t_total / reps
    flops = 2.0 * rows * case.k * case.n
    byts = rows * case.k * 2 + case.n * case.k + case.n * 4 + rows * case.n * 2
    return per, flops, byts, threads, rows, reps


def run_reference(args):
    """--impl reference: the CPU path timed on this box's host cores, on the same metric."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    case = make_case(args.workload)
    metric, unit = metric_of(case)
    per, flops, byts, threads, rows, reps = cpu_baseline(case, steps=max(args.steps, 1), warmup=max(args.warmup, 0))
    value = (byts / per / 1e9) if unit == "GB/s" else (flops / per / 1e12)
    sample = (f"{rows} of {case.m} rows per step ({reps} steps timed after {args.warmup} untimed), full weight "
              f"dequantized each step (oracle/ C, OpenMP) + fp32 torch.matmul on the CPU")
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": reps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
            "scaling": "strong" if (world > 1 and args.workload == "cfg1") else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": describe(case, args.workload, world),
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    from siliconed_b200.products import Context, QuantizedWeight

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    case = make_case(args.workload)
    metric, unit = metric_of(case)
    # cfg1-w8a8: config 1's data through the W8A8 route (x quantized to int8 per row, int8 x int8 on the
    # tensor cores): another arithmetic than config 1's weight-only product, reported beside it.
    w8a8 = args.workload.endswith("-w8a8")
    if w8a8:
        metric, unit = "W8A8 (int8 activation x int8 weight) GEMM TOP/s at M=4096", "TOP/s"
    ctx = Context(local)
    w = QuantizedWeight(ctx, case.codes_nk, case.kind, case.scales, published_nk=True)
    x = torch.from_numpy(case.x.view(np.int16)).cuda().view(torch.bfloat16)
    bias = None if case.bias is None else torch.from_numpy(case.bias.view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty((case.m, case.n), dtype=torch.bfloat16, device="cuda")
    ws_bytes = w.w8a8_workspace_bytes(case.m) if w8a8 else w.workspace_bytes(case.m)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    clean = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")

    def flush_l2(i):
        # A write larger than the L2 evicts the inputs; a read of another buffer larger than the L2 then
        # replaces the written (dirty) lines with clean ones, so that their write-back does not land in
        # the next timed step.
        flush.fill_(i & 0xFF)
        torch.sum(clean, dim=0, out=sink)
    stream = torch.cuda.current_stream()

    def step():
        if w8a8:
            w.linear_w8a8(x, y, bias=bias, workspace=ws, stream=stream)
        else:
            w.linear(x, bias=bias, out=y, workspace=ws, stream=stream)

    for _ in range(args.warmup):
        flush_l2(1)
        step()
    ctx.poll_errors()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        # The device sleeps while the host enqueues every step, so that the events around each
        # product measure the device's execution of it, not the host's launch overhead (the e2e
        # figure below measures the public call itself).
        torch.cuda._sleep(int(2e6) * max(1, args.steps // 10))
        for i in range(args.steps):
            flush_l2(i)
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ctx.poll_errors()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]  # ms
    t_ms = float(sum(per_step))
    t = torch.tensor([t_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_ms = float(t.item())
    sec_per_step = t_ms / 1e3 / args.steps
    value = throughput(case, sec_per_step, unit, ranks=world)

    # End to end through the public API with host buffers: every step copies x in from pinned host memory,
    # multiplies and copies y back (sc_linear_host: the rows in chunks, copies overlapped with products).
    x_host = torch.from_numpy(case.x.view(np.int16)).view(torch.bfloat16).pin_memory()
    y_host = torch.empty((case.m, case.n), dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)
    e2e_steps = max(3, min(args.steps, 20))
    # y goes through a device buffer and chunked copies back (the products writing the pinned y themselves,
    # sc_linear_host's direct mode, measured slower: 97 against 104 TFLOP/s end to end for config 1).
    direct_out = False

    def e2e_step():
        if w8a8:   # copy in, product, copy out on one stream
            x_dev.copy_(x_host, non_blocking=True)
            w.linear_w8a8(x_dev, y, bias=bias, workspace=ws, stream=stream)
            y_host.copy_(y, non_blocking=True)
        else:
            w.linear_host(x_host, y_host, bias=bias, x_dev=x_dev, y_dev=None if direct_out else y, workspace=ws,
                          stream=stream, direct=direct_out)
    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        dist.barrier()
    e2e_value = throughput(case, float(te.item()) / 1e3 / e2e_steps, unit, ranks=world)

    # Yardstick (one GPU, the GEMM configs): cuBLAS through torch.matmul, bf16 x . bf16 W on the same shape, the
    # weight dequantized and rounded to bf16, no scale and no bias, in the same harness (L2 flushed, events
    # around each step).  A library GEMM on a plain bf16 weight: what this shape gives without quantization.
    yardstick = None
    if world == 1 and unit != "GB/s" and not w8a8:
        wb = w.dequantize().to(torch.bfloat16)
        yb = torch.empty((case.m, case.n), dtype=torch.bfloat16, device="cuda")
        for _ in range(args.warmup):
            flush_l2(1)
            torch.matmul(x, wb, out=yb)
        ys = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ye = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        torch.cuda.synchronize()
        torch.cuda._sleep(int(2e6) * max(1, args.steps // 10))
        for i in range(args.steps):
            flush_l2(i)
            ys[i].record(stream)
            torch.matmul(x, wb, out=yb)
            ye[i].record(stream)
        torch.cuda.synchronize()
        y_ms = sum(a.elapsed_time(b) for a, b in zip(ys, ye)) / args.steps
        yardstick = {"what": "torch.matmul (cuBLAS) bf16 x [M, K] . W [K, N], W dequantized and rounded to bf16, "
                             "no scale or bias; same L2 flush and events",
                     "ms_per_step": y_ms, "value": case.flops / (y_ms / 1e3) / 1e12, "unit": "TFLOP/s"}
        del wb, yb

    if rank == 0:
        peaks, peak_src = load_peaks()
        if unit == "GB/s":
            achieved = case.bytes_moved() / sec_per_step / 1e9
            peak, runit, bound = peaks["hbm_gbs"], "GB/s", "hbm"
        elif w8a8:
            achieved = case.flops / sec_per_step / 1e12
            peak, runit, bound = 2.0 * peaks["bf16_tflops"], "TOP/s", "tensor"
        else:
            achieved = case.flops / sec_per_step / 1e12
            peak, runit, bound = peaks["bf16_tflops"], "TFLOP/s", "tensor"
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.txt")
        if os.path.exists(tpath):
            for line in open(tpath):
                parts = line.split()
                if len(parts) == 2 and not line.startswith("#") and parts[0] == args.workload:
                    traffic = int(parts[1])
        line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8" if w8a8 else "bf16", "data": "synthetic",
                "config": describe(case, args.workload, world),
                "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": runit,
                             "frac": achieved / peak, "traffic": traffic,
                             "peak_source": f"{peak_src} (burst figure: the kernel is timed alone)",
                             "kernels": (["sign_codes", "quantize_rows", "gemm_bf16_pair (kind::i8)"] if w8a8
                                         else route_kernels(case, ws_bytes))},
                "clocks": clocks.summary(),
                "e2e": {"value": e2e_value, "unit": unit,
                        "h2d_bytes_per_step": int(case.x.nbytes),
                        "d2h_bytes_per_step": int(case.m * case.n * 2),
                        "path": "QuantizedWeight.linear_host (sc_linear_host): pinned host x in, y out, every step; "
                                "x copied in chunks of rows overlapped with the products"
                                + ("; the products write the pinned y themselves" if direct_out else
                                   "; y copied back in chunks")},
                "gpu_launches": args.steps * (3 if w8a8 else len(route_kernels(case, ws_bytes))),
                "step_ms_min": min(per_step), "step_ms_median": statistics.median(per_step)}
        if yardstick is not None:
            line["yardstick"] = yardstick
        if w8a8:
            line["roofline"]["peak_source"] += "; int8 dense peak taken as 2 x the measured bf16 figure (the nominal ratio)"
            line["e2e"]["path"] = "QuantizedWeight.linear_w8a8 with pinned host x in and y out on one stream, every step"
        if not args.no_cpu_baseline and world == 1 and not w8a8:
            per, flops, byts, threads, rows, reps = cpu_baseline(case)
            cv = (byts / per / 1e9) if unit == "GB/s" else (flops / per / 1e12)
            line["cpu_baseline"] = {"value": cv, "unit": unit, "cores": threads, "kind": "port",
                                    "sample": f"{rows} of {case.m} rows, {reps} reps: oracle dequant (C, OpenMP) "
                                              f"+ fp32 torch.matmul, {per * 1e3:.1f} ms each"}
        print(json.dumps(line), flush=True)
    w.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


CHAIN_LAYERS = 8


def run_chain(args):
    """chainM (M = 1, 4, 16, 32): the decode case of config 4 as a model runs it, eight distinct int8 weights
    back to back, [12288 out, 4096 in] and [4096 out, 12288 in] alternating (an MLP's up and down products),
    each layer's bf16 output the next one's input; every weight is read cold (400 MB in all, beyond the L2),
    the L2 flushed once before each chain.  A step is one pass through the eight layers; value: the chain's
    algorithmic bytes (every weight, scale, input and output once) over its time, per second."""
    import torch
    from siliconed_b200 import configs
    from siliconed_b200.products import Context, QuantizedWeight

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(local)
    m = int(args.workload[5:])
    ctx = Context(local)
    shapes = [(12288, 4096), (4096, 12288)] * (CHAIN_LAYERS // 2)
    cases = [configs.config4(m, n, k, seed=i) for i, (n, k) in enumerate(shapes)]
    weights = [QuantizedWeight(ctx, c.codes_nk, c.kind, c.scales, published_nk=True) for c in cases]
    acts = [torch.from_numpy(cases[0].x.view(np.int16)).cuda().view(torch.bfloat16)]
    for n, _ in shapes:
        acts.append(torch.empty((m, n), dtype=torch.bfloat16, device="cuda"))
    ws_need = max(w.workspace_bytes(m) for w in weights)
    ws = torch.empty(max(ws_need, 1), dtype=torch.uint8, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    clean = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    chain_bytes = sum(c.bytes_moved() for c in cases)

    def step():
        for i, w in enumerate(weights):
            w.linear(acts[i], out=acts[i + 1], workspace=ws, stream=stream)

    for _ in range(args.warmup):
        flush.fill_(1)
        torch.sum(clean, dim=0, out=sink)
        step()
    ctx.poll_errors()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        torch.cuda._sleep(int(2e6) * max(1, args.steps // 5))
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            torch.sum(clean, dim=0, out=sink)
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    ctx.poll_errors()
    per = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    ms = sum(per) / len(per)
    value = chain_bytes / (ms / 1e3) / 1e9
    # the first two layers one at a time, each after its own flush (the single cold read)
    single = []
    for i, w in enumerate(weights[:2]):
        ev = []
        for r in range(max(args.steps, 3)):
            flush.fill_(r & 0xFF)
            torch.sum(clean, dim=0, out=sink)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            w.linear(acts[i], out=acts[i + 1], workspace=ws, stream=stream)
            b.record(stream)
            ev.append((a, b))
        torch.cuda.synchronize()
        t = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
        single.append({"shape": list(shapes[i]), "us": t * 1e3, "gb_s": cases[i].bytes_moved() / (t / 1e3) / 1e9})
    if rank == 0:
        peaks, peak_src = load_peaks()
        kern = route_kernels(cases[0], ws_need)
        line = {"metric": "int8-weight GEMV achieved HBM GB/s (decode chain, per layer)", "value": value,
                "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic",
                "config": {"workload": f"{args.workload}: {CHAIN_LAYERS} distinct int8 per-channel weights, "
                                       f"[12288, 4096] and [4096, 12288] alternating, x bf16 [{m}, K], each "
                                       f"output the next input", "m": m, "layers": CHAIN_LAYERS,
                           "bytes_per_chain": chain_bytes,
                           "l2": "flushed once before each chain (400 MB of weights, beyond the L2)",
                           "parallelism": "one GPU"},
                "roofline": {"bound": "hbm", "achieved": value, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": value / peaks["hbm_gbs"], "traffic": None, "peak_source": peak_src,
                             "kernels": kern},
                "single_cold_read": single, "clocks": clocks.summary(),
                "gpu_launches": args.steps * CHAIN_LAYERS * len(kern),
                "step_ms_min": min(per), "step_ms_median": statistics.median(per)}
        print(json.dumps(line), flush=True)
    for w in weights:
        w.close()
    ctx.close()
    return 0


def run_scale(args):
    """Config 1 on N > 1 GPUs, the default workload there (strong scaling: the total work is config 1's one
    product whatever N is).  Rank r registers W's columns column_ranges(N, P)[r] and multiplies the whole x
    by them; the product's epilogue stores every output tile into every rank's y over NVLink and raises an
    epoch flag on each rank, and a bounded wait kernel holds each rank's stream until all columns have
    landed (FusedColumnParallelLinear, sc_linear_allgather).  A step is one such call: widen, gathering GEMM,
    wait.  Before timing, every rank checks its gathered y against a single-GPU product of the whole weight,
    bit for bit ("parity").  The stores go to the peers' outputs opened through CUDA IPC; --multicast sends
    one multimem store per piece to the outputs' NVLink multicast address instead (torch symmetric memory).
    value: 77.31 GFLOP over the slowest rank's time per step."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from siliconed_b200 import configs, parallel
    from siliconed_b200.products import Context, QuantizedWeight

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    case = configs.config1()
    metric, unit = metric_of(case)
    ctx = Context(local)
    x = torch.from_numpy(case.x.view(np.int16)).cuda().view(torch.bfloat16)
    bias = torch.from_numpy(case.bias.view(np.int16)).cuda().view(torch.bfloat16)
    fused = parallel.FusedColumnParallelLinear(ctx, case.codes_nk, case.kind, case.scales, case.n, case.m,
                                               published_nk=True, bias=bias, multicast=args.multicast)
    stream = torch.cuda.current_stream()

    # parity, once: the gathered y of every rank against one GPU's product of the whole weight
    full = QuantizedWeight(ctx, case.codes_nk, case.kind, case.scales, published_nk=True)
    ws_full = torch.empty(max(full.workspace_bytes(case.m), 1), dtype=torch.uint8, device="cuda")
    y_ref = full.linear(x, bias=bias, workspace=ws_full)
    y_got = fused(x).clone()
    torch.cuda.synchronize()
    ctx.poll_errors()
    same = torch.tensor([1 if torch.equal(y_got.view(torch.int16), y_ref.view(torch.int16)) else 0],
                        dtype=torch.int32, device="cuda")
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    parity = bool(same.item() == 1)
    full.close()
    del y_ref, y_got, ws_full

    y_local = torch.empty((case.m, fused.n1 - fused.n0), dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    clean = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")

    def flush_l2(i):
        flush.fill_(i & 0xFF)
        torch.sum(clean, dim=0, out=sink)

    def step():
        fused(x)

    def product_alone():
        fused.w.linear(x, bias=fused.bias, out=y_local, workspace=fused.ws, stream=stream)

    def timed(fn, clocks=None):
        for i in range(args.warmup):
            flush_l2(1)
            fn()
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        dist.barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(int(2e6) * max(1, args.steps // 10))
        for i in range(args.steps):
            flush_l2(i)
            starts[i].record(stream)
            fn()
            ends[i].record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        per = [a.elapsed_time(b) for a, b in zip(starts, ends)]
        t = torch.tensor([sum(per)], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) / args.steps, per

    with ClockSampler(local) as clocks:
        ms_step, per_step = timed(step)
    ms_alone, _ = timed(product_alone)
    ctx.poll_errors()

    # End to end through the public call: x from pinned host memory, the fused product and gather, y back.
    x_host = torch.from_numpy(case.x.view(np.int16)).view(torch.bfloat16).pin_memory()
    y_host = torch.empty((case.m, case.n), dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        y = fused(x_dev)
        y_host.copy_(y, non_blocking=True)
    for _ in range(2):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 20))
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    dist.barrier()
    ctx.poll_errors()

    if rank == 0:
        peaks, peak_src = load_peaks()
        value = case.flops / (ms_step / 1e3) / 1e12
        width = max(b - a for a, b in fused.ranges)
        bytes_in = case.m * (case.n - width) * 2             # y's columns that arrive from the other ranks
        nvlink_gbs = 770.0                                   # measured peer copy per direction per GPU
        t_tensor = case.flops / world / (peaks["bf16_tflops"] * 1e12)
        t_link = bytes_in / (nvlink_gbs * 1e9)
        target_ms = 1e3 * max(t_tensor, t_link)
        line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": describe(case, args.workload, world),
                "parity": parity,
                "parity_check": "before timing, every rank's gathered y [4096, 3072] equal bit for bit to one "
                                "GPU's product of the whole weight",
                "collective": {"path": ("multicast stores (multimem.st to the outputs' NVLink multicast address)"
                                        if fused.uses_multicast else "peer stores over NVLink (CUDA IPC)"),
                               "columns_per_rank": width, "product_alone_us": ms_alone * 1e3,
                               "with_gather_us": ms_step * 1e3, "gather_extra_us": (ms_step - ms_alone) * 1e3,
                               "bytes_into_each_gpu": bytes_in,
                               "gb_s_into_each_gpu": bytes_in / (ms_step / 1e3) / 1e9},
                "roofline": {"bound": "tensor" if t_tensor >= t_link else "nvlink",
                             "achieved": value / world, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": value / world / peaks["bf16_tflops"], "traffic": None,
                             "peak_source": f"{peak_src} (burst figure)",
                             "fused_target_us": target_ms * 1e3, "frac_of_fused_target": target_ms / ms_step,
                             "target": "max(FLOPs per GPU / measured bf16 peak, bytes into each GPU / 770 GB/s "
                                       "measured peer copy)"},
                "clocks": clocks.summary(),
                "e2e": {"value": case.flops / (float(te.item()) / 1e3 / e2e_steps) / 1e12, "unit": unit,
                        "h2d_bytes_per_step": int(case.x.nbytes), "d2h_bytes_per_step": int(case.m * case.n * 2),
                        "path": "FusedColumnParallelLinear (sc_linear_allgather + sc_allgather_wait) with x copied "
                                "in from pinned host memory and the gathered y copied back, every step, every rank"},
                "gpu_launches": args.steps * 3,
                "step_ms_min": min(per_step), "step_ms_median": statistics.median(per_step)}
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    fused.close()
    ctx.close()
    dist.destroy_process_group()
    return 0


def run_colpar(args):
    """cfg1-colpar: config 1 with the weight's columns split over the ranks (sc_weight_create_shard), every
    rank multiplying the whole x by its columns, then one NCCL all-gather assembling y [M, N] on every rank.
    value: the whole product's TFLOP/s with the gather (the slowest rank's time); the line also carries the
    rate without it (strong scaling: the total work is fixed)."""
    import torch
    import torch.distributed as dist
    from siliconed_b200 import configs, parallel
    from siliconed_b200.products import Context, QuantizedWeight

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    case = configs.config1()
    ranges = parallel.column_ranges(case.n, world)
    n0, n1 = ranges[rank]
    ctx = Context(local)
    w = QuantizedWeight(ctx, case.codes_nk, case.kind, case.scales, published_nk=True, columns=(n0, n1))
    x = torch.from_numpy(case.x.view(np.int16)).cuda().view(torch.bfloat16)
    bias = torch.from_numpy(case.bias.view(np.int16)).cuda().view(torch.bfloat16)[n0:n1].contiguous()
    y_local = torch.empty((case.m, n1 - n0), dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(max(w.workspace_bytes(case.m), 1), dtype=torch.uint8, device="cuda")
    width = max(b - a for a, b in ranges)
    blocks = torch.empty((world * case.m, width), dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def product():
        w.linear(x, bias=bias, out=y_local, workspace=ws)

    def gather():
        if world > 1:
            dist.all_gather_into_tensor(blocks, y_local if y_local.shape[1] == width else
                                        torch.nn.functional.pad(y_local, (0, width - y_local.shape[1])))

    def timed(fn_list):
        for i in range(args.warmup):
            flush.fill_(1)
            for fn in fn_list:
                fn()
        st = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        en = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            st[i].record()
            for fn in fn_list:
                fn()
            en[i].record()
        torch.cuda.synchronize()
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(st, en)) / args.steps], dtype=torch.float64,
                         device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    fused = fused_mc = None
    if world > 1:
        bias_dev = torch.from_numpy(case.bias.view(np.int16)).cuda().view(torch.bfloat16)
        fused = parallel.FusedColumnParallelLinear(ctx, case.codes_nk, case.kind, case.scales, case.n, case.m,
                                                   published_nk=True, bias=bias_dev, multicast=False)
        fused_mc = parallel.FusedColumnParallelLinear(ctx, case.codes_nk, case.kind, case.scales, case.n, case.m,
                                                      published_nk=True, bias=bias_dev, multicast=True)
        if not fused_mc.uses_multicast:
            fused_mc.close()
            fused_mc = None
    with ClockSampler(local) as clocks:
        ms_gather = timed([product, gather])
        ms_local = timed([product])
        ms_fused = timed([lambda: fused(x)]) if fused is not None else None
        ms_fused_mc = timed([lambda: fused_mc(x)]) if fused_mc is not None else None
    ctx.poll_errors()
    if rank == 0:
        peaks, peak_src = load_peaks()
        value = case.flops / (ms_gather / 1e3) / 1e12
        line = {"metric": "int8-weight GEMM TFLOP/s at M=4096 (column-parallel, with the all-gather)", "value": value,
                "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_gather, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "cfg1-colpar: config 1, W's columns split over the ranks, y all-gathered (NCCL)",
                           "m": case.m, "k": case.k, "n": case.n, "columns_per_rank": width,
                           "parallelism": f"column-parallel x{world}"},
                "without_gather": {"value": case.flops / (ms_local / 1e3) / 1e12, "ms_per_step": ms_local},
                "fused_gather": (None if ms_fused is None else
                                 {"value": case.flops / (ms_fused / 1e3) / 1e12, "ms_per_step": ms_fused,
                                  "path": "sc_linear_allgather (product epilogue stores every tile to every rank "
                                          "over NVLink) + sc_allgather_wait"}),
                "fused_gather_multicast": (None if ms_fused_mc is None else
                                           {"value": case.flops / (ms_fused_mc / 1e3) / 1e12, "ms_per_step": ms_fused_mc,
                                            "path": "sc_linear_allgather_mc (one multimem store per piece to the outputs' "
                                                    "NVLink multicast address) + sc_allgather_wait"}),
                "gather_bytes_per_rank": int(case.m * width * 2 * (world - 1)),
                "roofline": {"bound": "tensor", "achieved": value / world, "peak": peaks["bf16_tflops"],
                             "unit": "TFLOP/s", "frac": value / world / peaks["bf16_tflops"], "traffic": None,
                             "peak_source": peak_src},
                "clocks": clocks.summary(), "gpu_launches": args.steps * (2 if case.m >= 1536 else 1)}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    if fused is not None:
        fused.close()
    if fused_mc is not None:
        fused_mc.close()
    w.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


DIT_WORKLOADS = ("cfg3", "cfg5")
ATTN_SHAPES = {"attn3": (1, 30, 4608), "attn5": (8, 24, 4352)}  # [batch, heads, joint tokens], head_dim 128


def run_attention(args):
    """attn3 / attn5: the attention of config 3 (1 x 30 heads x 4608 tokens) or config 5 (8 images x 24 heads x
    4352 joint tokens) alone, sd_attention on bf16 q, k, v [B, H, S, 128] (seeded N(0, 1)), with torch's fused
    SDPA on the same inputs timed beside it as the yardstick.  value: 4 B H S^2 128 FLOP over the device time of
    one call; the inputs (141 MB / 580 MB) exceed the L2, and the L2 is flushed before every step anyway."""
    import torch
    from siliconed_b200 import dit_abi

    b, h, s = ATTN_SHAPES[args.workload]
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(b, h, s, 128, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    flops = 4.0 * b * h * s * s * 128
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(args.warmup):
            flush.fill_(1)
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        torch.cuda._sleep(int(2e6))
        for i, (a, e) in enumerate(ev):
            flush.fill_(i & 0xFF)
            a.record(stream)
            fn()
            e.record(stream)
        torch.cuda.synchronize()
        per = [a.elapsed_time(e) for a, e in ev]
        return sum(per) / len(per), per

    with ClockSampler(0) as clocks:
        ms, per = timed(lambda: dit_abi.attention(q, k, v, o, 1.0 / math.sqrt(128)))
    status = dit_abi.attention_errors()
    if status != (0, 0):
        raise SystemExit(f"sd_attention: a bounded wait gave up {status}")
    ms_lib, _ = timed(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v))
    peaks, peak_src = load_peaks()
    value = flops / (ms / 1e3) / 1e12
    line = {"metric": "attention TFLOP/s (head_dim 128, bf16)", "value": value, "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.workload}: softmax(q k^T / sqrt(128)) v, q, k, v, o bf16 [{b}, {h}, {s}, 128]",
                       "batch": b, "heads": h, "seq": s, "l2": "flushed before every timed step",
                       "parallelism": "one GPU"},
            "roofline": {"bound": "tensor", "achieved": value, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": value / peaks["bf16_tflops"], "traffic": None,
                         "peak_source": f"{peak_src} (burst figure)", "kernels": ["attention_fwd"]},
            "yardstick": {"what": "torch.nn.functional.scaled_dot_product_attention on the same bf16 inputs",
                          "ms_per_step": ms_lib, "value": flops / (ms_lib / 1e3) / 1e12, "unit": "TFLOP/s"},
            "clocks": clocks.summary(), "gpu_launches": args.steps,
            "step_ms_min": min(per), "step_ms_median": statistics.median(per)}
    print(json.dumps(line), flush=True)
    return 0


def dit_cpu_seconds(shapes, rows_full: int, rows_sample: int = 256):
    """The reference's CPU route for one block's linears (oracle dequantization of each weight, C with
    OpenMP over all host threads, then an fp32 torch.matmul), timed on `rows_sample` rows and scaled
    to `rows_full`; returns (seconds per block, threads)."""
    import torch
    import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    torch.set_num_threads(threads)
    rng = np.random.default_rng(0)
    total = 0.0
    for k, n in shapes:
        q = rng.integers(-127, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        sc = np.full(n, 1e-3, np.float32)
        x = torch.randn(rows_sample, k)
        t0 = time.perf_counter()
        w = oracle.dequantize(q, 1, sc, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
        t1 = time.perf_counter()
        x @ torch.from_numpy(w)
        t2 = time.perf_counter()
        total += (t1 - t0) + (t2 - t1) * rows_full / rows_sample
    return total, threads


def run_dit(args):
    """Configs 3 and 5 (the DiT block and the 8-step MMDiT denoise) over the quantized linears.

    cfg3: a step is one forward of one single-stream block (S = 4096 image + 512 text tokens, d 3840);
    metric TFLOP/s of its linears and attention.  cfg5: a step is one denoise step (one forward of the
    60-block MMDiT over the batch); the batch of 8 images is split across the ranks (strong scaling);
    metric s/image of the 8-step denoise = 8 x (slowest rank's time per step) / 8 images."""
    import torch
    import torch.distributed as dist
    from siliconed_b200 import dit
    from siliconed_b200.products import Context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    ctx = Context(local)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    if args.workload == "cfg3":
        s_img, s_txt, d = 4096, 512, 3840
        s = s_img + s_txt
        model = dit.ZImageBlock(ctx, dim=d, heads=30, hidden=10240, seed=0)
        x0 = torch.randn(s, d, generator=g, device="cuda")
        x = x0.clone()
        grid = int(round(s_img ** 0.5))
        freqs = dit.rope_table(dit.image_text_positions(s_txt, grid)).cuda()
        adaln = dit.timestep_embedding(0.5)
        flops = model.flops(s)

        def step(i):
            x.copy_(x0)
            model.forward(x, freqs, adaln)
        images = None
        metric, unit, hib = "DiT block (config 3) TFLOP/s", "TFLOP/s", True
        launches_per_step = 15
        cpu_shapes = [(d, 3 * d), (d, d), (d, 2 * 10240), (10240, d), (256, 4 * d)]
        cpu_rows = s
        config = {"workload": "cfg3: one single-stream DiT block, 4096 image + 512 text tokens, d 3840, 30 x 128 heads, "
                              "SwiGLU 10240, adaLN 256 -> 4 d; int8 per-channel linears (N(0, 0.02) random init)",
                  "tokens": s, "dim": d, "heads": 30, "hidden": 10240, "batch": 1}
    else:
        batch_total, st, si, d = 8, 256, 4096, 3072
        if batch_total % world != 0:
            raise SystemExit(f"cfg5: {world} ranks do not divide the batch of {batch_total}")
        batch = batch_total // world
        blocks = int(os.environ.get("SC_MMDIT_BLOCKS", "60"))
        model = dit.MMDiT(ctx, blocks=blocks, dim=d, heads=24, mlp=12288, seed=0)
        z = torch.randn(batch * si, 64, generator=g, device="cuda")
        txt = (torch.randn(batch * st, d, generator=g, device="cuda")).to(torch.bfloat16)
        freqs = dit.rope_table(dit.image_text_positions(st, 64)).cuda()
        sig = torch.linspace(1.0, 0.0, 9).tolist()

        def step(i):
            v = model.forward(z, txt, batch, sig[i % 8], freqs)
            z.add_(v, alpha=sig[i % 8 + 1] - sig[i % 8])
        flops = model.flops_per_step(batch, st, si)
        images = batch_total
        metric, unit, hib = "DiT s/image 1024x1024 8-step (MMDiT, 60 double-stream blocks, batch 8)", "s/image", False
        launches_per_step = None
        cpu_shapes = [(256, 6 * d), (d, 3 * d), (d, d), (d, 12288), (12288, d)]
        cpu_rows = batch_total * (st + si)
        config = {"workload": f"cfg5: {blocks} double-stream MMDiT blocks, d 3072, 24 x 128 heads, MLP 12288 GELU (tanh), "
                              f"4096 image + 256 text tokens, batch 8 ({batch} per rank), 8 Euler steps; int8 per-channel "
                              f"linears (N(0, 0.02) random init), {model.weight_bytes() / 1e9:.1f} GB of weights per GPU",
                  "blocks": blocks, "dim": d, "heads": 24, "mlp": 12288, "batch": batch_total, "batch_per_rank": batch,
                  "steps_per_image": 8}

    for i in range(args.warmup):
        flush.fill_(1)
        step(i)
    torch.cuda.synchronize()
    ctx.poll_errors()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            starts[i].record()
            step(i)
            ends[i].record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ctx.poll_errors()
    per_step = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    t = torch.tensor([sum(per_step)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    tflops_rank = flops / (ms_per_step / 1e3) / 1e12
    if images is None:
        value = world * tflops_rank
    else:
        value = 8 * ms_per_step / 1e3 / images  # 8 steps of the whole batch, per image

    # End to end through the public call: latents / activations from pinned host memory, the result back.
    if args.workload == "cfg3":
        host_in = x0.cpu().pin_memory()
        host_out = torch.empty_like(host_in).pin_memory()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        x.copy_(host_in, non_blocking=True)
        model.forward(x, freqs, adaln)
        host_out.copy_(x, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        te = e0.elapsed_time(e1)
        e2e = {"value": world * flops / (te / 1e3) / 1e12, "unit": unit, "h2d_bytes_per_step": host_in.numel() * 4,
               "d2h_bytes_per_step": host_in.numel() * 4, "path": "ZImageBlock.forward with x from pinned host memory"}
    else:
        z_host = z.cpu().pin_memory()
        t_host = txt.cpu().pin_memory()
        out_host = torch.empty_like(z_host).pin_memory()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        z.copy_(z_host, non_blocking=True)
        txt.copy_(t_host, non_blocking=True)
        model.denoise(z, txt, batch, 8, freqs)
        out_host.copy_(z, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": float(te.item()) / 1e3 / images, "unit": unit,
               "h2d_bytes_per_step": (z_host.numel() * 4 + t_host.numel() * 2) // 8,
               "d2h_bytes_per_step": z_host.numel() * 4 // 8,
               "path": "MMDiT.denoise (8 steps) with latents and text from pinned host memory, latents back"}

    if rank == 0:
        peaks, peak_src = load_peaks()
        line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": hib,
                "scaling": "strong" if images is not None else "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init weights of the architecture, N(0,1) latents and activations)",
                "config": config,
                "roofline": {"bound": "tensor", "achieved": tflops_rank, "peak": peaks["bf16_tflops_sustained"],
                             "unit": "TFLOP/s", "frac": tflops_rank / peaks["bf16_tflops_sustained"], "traffic": None,
                             "peak_source": f"{peak_src} (sustained figure: a long step)",
                             "note": "achieved = the step's linear and attention FLOPs per rank over the step's time"},
                "clocks": clocks.summary(), "e2e": e2e,
                "gpu_launches": (args.steps * launches_per_step if launches_per_step else None),
                "step_ms_min": min(per_step), "step_ms_median": statistics.median(per_step)}
        if images is not None:
            line["gpu_launches"] = args.steps * dit_launches_per_step(model)
        if not args.no_cpu_baseline and world == 1:
            per_block, threads = dit_cpu_seconds(cpu_shapes, cpu_rows)
            if images is None:
                cv = flops / per_block / 1e12
                sample = "one block's linears: 256 of 4608 rows timed, scaled to 4608 (attention not included)"
            else:
                per_block *= 2  # two streams
                cv = per_block * len(model.blocks) * 8 / images
                sample = ("one double-stream block's linears (both streams) on 256 of 34816 rows, scaled to the batch, "
                          "x 60 blocks x 8 steps / 8 images (extrapolated; attention not included)")
            line["cpu_baseline"] = {"value": cv, "unit": unit, "cores": threads, "kind": "port", "sample": sample}
        print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def dit_launches_per_step(model) -> int:
    """This project's kernels in one MMDiT forward (the attention is the CUDA library's and not counted):
    per stream and block the modulation GEMV, two LayerNorms, QK-norm + RoPE, GELU, two residuals and
    four products (two launches each where the widened route runs, i.e. from 1536 rows)."""
    blocks = len(model.blocks)
    b = model._bufs[0] if model._bufs else None
    batch, st, si = b if b else (8, 256, 4096)
    def prod(m):
        return 2 if m >= 1536 else 1
    per_stream = lambda m: 1 + 2 + 1 + 1 + 2 + 4 * prod(m)
    return blocks * (per_stream(batch * st) + per_stream(batch * si)) + prod(batch * si) * 2 + prod(batch * st) + 2


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--multicast", action="store_true",
                    help="N > 1: the gathered stores go to an NVLink multicast address (default: peer stores)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.workload == "cfg1-colpar" and args.impl == "ours":
        return run_colpar(args)
    if args.workload == "cfg1" and args.impl == "ours" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_scale(args)
    if args.workload.startswith("chain") and args.impl == "ours":
        return run_chain(args)
    if args.workload in ATTN_SHAPES:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the attention workloads have no CPU reference arm "
                              "(the yardstick on the ours line is the library's GPU attention)"}), flush=True)
            return 0
        return run_attention(args)
    if args.workload in DIT_WORKLOADS:
        if args.impl == "reference":
            rank = int(os.environ.get("RANK", "0"))
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the DiT workloads' reference arm is the "
                                  "CPU extrapolation reported as cpu_baseline on the ours line"}), flush=True)
            return 0
        return run_dit(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
