#!/usr/bin/env python3
"""Benchmark of the kvbridge-b200 decode-attention path (one JSON line).

Headline workload (BASELINE cfg2): one decode call per step - batch 1,
65,536-token context, 32 query / 8 KV heads, head dim 128, INT8 K/V with
per-(token, head) fp32 scales, 64-token pages shuffled, fp16 N(0,1) queries,
split-K partitions chosen by the launcher, fp16 output. Inputs are seeded
synthetic data with BASELINE's value distributions.

At N GPUs (torchrun, one rank per GPU) the headline is the SAME problem split
over the ranks along KV heads (rank g owns KV heads [8g/N, 8(g+1)/N) and their
query heads; no collective on the data path): strong scaling, value = the
problem's KV bytes / the slowest rank's time per call. Two more keys:
  * weak_replicated - every rank runs a whole cfg2 (8 KV heads of a model
    with 8N), value = N x bytes / the slowest rank's time per call;
  * cfg5_sequence_sharded - BASELINE cfg5 (4 sequences x 1,048,576 tokens)
    split along the sequence: each rank decodes its page-aligned range of
    every sequence (batched call), writes its (m, l, n) partial into one
    packed buffer, the buffers are all-gathered in ONE NCCL collective and
    merged by merge_attention_shards_ex, all inside the timed region.

Timing: steps are replayed from CUDA graphs that hold a whole number of
--steps-step blocks (>= --block-calls calls); the timed region repeats whole
graph replays until it covers --min-seconds (>= 1 s), bracketed by a barrier
and cuda synchronize, timed with CUDA events between replays on the launching
stream; the time per call is the median over replays, max over ranks. Each
step reads another of the resident KV "layers" (>= 553 MB in total, > 4x the
126 MB L2), so no step finds its KV in L2. Clocks are sampled with nvidia-smi
over exactly the headline's timed window.

Metric: effective KV GB/s = algorithmic KV bytes (int8 K + V + fp32 K/V
scales of every attended token and KV head: 2,112 B/token at 8 x 128) per
call / time per call; ms_per_step is the time per call.

`--impl reference` times the reference's own CPU implementation (its FP64
oracle compiled from its sources into oracle/_ref; the C restatement in
oracle/ when that build is absent) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# Steps per group in the end-to-end leg: the call stream waits on the copy
# streams once per group instead of once per step.
E2E_GROUP = 50
METRIC = "µs/decode-attention call and effective KV GB/s (% of HBM peak) at 64K ctx, 1–8 B200"
WORKLOAD = dict(
    workload="cfg2: single-layer decode attention, 65,536 ctx",
    batch=1,
    context=65536,
    q_heads=32,
    kv_heads=8,
    head_dim=128,
    page_tokens=64,
    kv_dtype="int8 + fp32 per-(token, kv-head) scales",
    q_dtype="fp16 values (fp32 storage)",
    out_dtype="fp16",
)
SEED = 0xC0FFEE + 2
L2_BYTES = 126 * 1024 * 1024
RESIDENT_BYTES = 4 * 138_412_032  # KV bytes kept resident per timed leg (> 4x L2)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--partitions", type=int, default=0, help="split-K partitions per KV head (0 = auto)")
    ap.add_argument("--min-seconds", type=float, default=1.5, help="length of each timed region")
    ap.add_argument("--block-calls", type=int, default=500, help="calls per CUDA graph (rounded to whole step blocks)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the weak-scaling and cfg5 keys")
    ap.add_argument("--config", choices=["cfg2", "cfg1", "cfg3", "cfg4", "cfg5", "native", "f32"], default="cfg2",
                    help="BASELINE workload; the headline line is cfg2, the others are informational "
                         "(native: the reference MMA kernel's rows-8 / 24-4 heads / dim-256 / Page32 shape; "
                         "f32: cfg2's geometry with fp32 KV)")
    ap.add_argument("--kernel", choices=["auto", "warp", "tcgen05", "general"], default="auto",
                    help="single-sequence partial kernel (auto = chosen by shape; general = the CUDA-core "
                         "kernel for every call)")
    return ap.parse_args()


def kv_bytes_per_call(tokens: int, kv_heads: int, dim: int) -> int:
    return tokens * kv_heads * (2 * dim + 8)


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per partial-kernel launch at cfg2 from the committed ncu
    summary (profiles/decode_partial_cfg2.txt, line `traffic_bytes_per_launch:`)."""
    path = ROOT / "profiles" / "decode_partial_cfg2.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.


class ClockSampler:
    FIELDS = (
        "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu_id],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._pump, daemon=True)
        self.thread.start()

    def _pump(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, window=None):
        """Summary of the samples taken inside `window` (host times (t0, t1))."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for arrived, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            stamp = arrived
            try:
                stamp = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                pass
            if window is not None and not (window[0] <= stamp <= window[1]):
                continue
            try:
                sms.append(float(parts[2]))
                maxes.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sms) if sms else None,
            "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": sorted(reasons),
            "samples": len(sms),
        }


# ---------------------------------------------------------------------------
# CPU baselines (the reference's own oracle, or the C restatement).


def cpu_reference_runner(case_cpu, threads: int):
    import oracle

    if oracle.RefOracle.available():
        run = oracle.RefOracle().prepare(
            case_cpu.shape, case_cpu.q, case_cpu.q_positions, case_cpu.k_positions, case_cpu.page_table,
            case_cpu.k, case_cpu.v, case_cpu.k_scales, case_cpu.v_scales,
        )
        return "reference", (lambda: run.run(threads)), run

    def port():
        t0 = time.perf_counter()
        oracle.reference_case(case_cpu, threads=threads)
        return time.perf_counter() - t0

    return "port", port, None


def sample_case(tokens: int, device: str):
    from kvbridge_b200 import synth

    return synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=tokens,
                             seed=SEED, device=device)


def cpu_baseline(case_cpu, min_cpu_seconds: float = 10.0, max_calls: int = 20):
    threads = os.cpu_count() or 1
    kind, run, _keep = cpu_reference_runner(case_cpu, threads)
    times = []
    while len(times) < max_calls:
        times.append(run())
        if len(times) >= 2 and sum(times) * threads >= min_cpu_seconds:
            break
    per_call = statistics.median(times)
    gbs = kv_bytes_per_call(case_cpu.shape.end - case_cpu.shape.begin, 8, 128) / per_call / 1e9
    return {
        "value": round(gbs, 4),
        "unit": "GB/s",
        "cores": threads,
        "kind": kind,
        "sample": f"{len(times)} full cfg2 calls (65,536 tokens x 32 q-heads) on {threads} threads, "
                  f"median {per_call * 1e3:.1f} ms/call",
        "ms_per_call": round(per_call * 1e3, 3),
    }


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    steps, warmup = args.steps, args.warmup
    # Each step is a bounded sample: the full 32-head computation over a
    # contiguous token range sized so that warmup + steps take ~90 s.
    full = sample_case(65536, "cpu")
    import oracle

    kind = "reference" if oracle.RefOracle.available() else "port"
    # Calibrate the per-token cost on 4,096 tokens.
    calib_tokens = 4096
    cal = sample_case(65536, "cpu")
    cal.shape.begin, cal.shape.end = 65536 - calib_tokens, 65536
    _, run_cal, keep_cal = cpu_reference_runner(cal, threads)
    run_cal()
    t_cal = min(run_cal() for _ in range(2))
    per_token = t_cal / calib_tokens
    budget = 90.0
    tokens = int(min(65536, max(64, budget / max(1, steps + warmup) / per_token)))
    tokens = max(64, (tokens // 64) * 64)
    full.shape.begin, full.shape.end = 65536 - tokens, 65536
    _, run, keep = cpu_reference_runner(full, threads)
    for _ in range(warmup):
        run()
    times = [run() for _ in range(steps)]
    per_call = sum(times) / len(times)
    nbytes = kv_bytes_per_call(tokens, 8, 128)
    value = nbytes / per_call / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(per_call * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic (seeded; BASELINE cfg2 value distributions)",
        "config": dict(WORKLOAD, sample_tokens=tokens, l2="host CPU run"),
        "cpu_baseline": {
            "value": round(value, 4),
            "unit": "GB/s",
            "cores": threads,
            "kind": kind,
            "sample": f"each step: the last {tokens} of 65,536 tokens for all 32 q-heads "
                      f"({threads} threads, "
                      + ("the reference's FP64 CPU oracle built from its sources)" if kind == "reference"
                         else "the C restatement of the reference's FP64 oracle)"),
        },
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Timing: whole graph replays (or eager blocks) until the region is long.


class Bench:
    def __init__(self, args, world, rank, local_rank, device):
        import torch

        self.torch = torch
        self.args = args
        self.world, self.rank, self.local_rank, self.device = world, rank, local_rank, device
        self.stream = torch.cuda.Stream(device=device)
        self.steps = max(1, args.steps)
        self.block = self.steps * max(1, math.ceil(args.block_calls / self.steps))

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[self.local_rank])

    def max_over_ranks(self, values):
        torch = self.torch
        if self.world == 1:
            return list(values)
        import torch.distributed as dist

        t = torch.tensor(list(values), dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]

    def gather(self, value):
        torch = self.torch
        if self.world == 1:
            return [value]
        import torch.distributed as dist

        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        out = torch.empty(self.world, dtype=torch.float64, device=self.device)
        dist.all_gather_into_tensor(out, t)
        return [float(x) for x in out.tolist()]

    def capture(self, step, calls):
        """A CUDA graph of `calls` steps (step(i) enqueues call i)."""
        torch = self.torch
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            for i in range(calls):
                step(i)
        return g

    def timed(self, block_fn, calls_per_block, warmup_blocks=1, min_seconds=None, window=None):
        """Runs block_fn() (calls_per_block calls on self.stream) until the
        region covers min_seconds; returns the median time per call (max over
        ranks), the region's length and counts. `window`, when given, gets
        the host times bracketing the timed region."""
        torch = self.torch
        min_seconds = self.args.min_seconds if min_seconds is None else min_seconds
        with torch.cuda.stream(self.stream):
            for _ in range(max(1, warmup_blocks)):
                block_fn()
        torch.cuda.synchronize()
        # Calibrate the number of blocks (the same on every rank).
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            a.record(self.stream)
            block_fn()
            b.record(self.stream)
        torch.cuda.synchronize()
        t_block = max(a.elapsed_time(b), 1e-3) / 1e3
        blocks = int(self.max_over_ranks([min(100000, max(3, math.ceil(min_seconds / t_block)))])[0])
        events = [torch.cuda.Event(enable_timing=True) for _ in range(blocks + 1)]
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        t0 = time.time()
        with torch.cuda.stream(self.stream):
            events[0].record(self.stream)
            for i in range(blocks):
                block_fn()
                events[i + 1].record(self.stream)
        torch.cuda.synchronize()
        t1 = time.time()
        self.barrier()
        if window is not None:
            window[:] = [t0, t1]
        per_block = [events[i].elapsed_time(events[i + 1]) for i in range(blocks)]
        total_ms = events[0].elapsed_time(events[-1])
        med = statistics.median(per_block) / calls_per_block
        p95 = sorted(per_block)[int(0.95 * (blocks - 1))] / calls_per_block
        mean = total_ms / (blocks * calls_per_block)
        med_max, p95_max, mean_max, total_max = self.max_over_ranks([med, p95, mean, total_ms])
        return {"per_call_ms": med_max, "p95_per_call_ms": p95_max, "mean_per_call_ms": mean_max,
                "region_s": total_max / 1e3, "blocks": blocks, "calls": blocks * calls_per_block,
                "rank_per_call_ms": med}


def check_status(kvb, where):
    status = kvb.read_device_status()
    if status != 0:
        raise RuntimeError(f"{where}: kernel status word {status}: a bounded wait gave up or a page was bad "
                           f"({kvb.read_wait_failure()}); numbers invalid")


def make_layers(synth, world, rank, kv_heads, q_heads, device):
    per_layer = kv_bytes_per_call(65536, kv_heads, 128)
    count = max(4, math.ceil(RESIDENT_BYTES / per_layer))
    return [synth.make_single(rows=1, q_heads=q_heads, kv_heads=kv_heads, dim=128, page_tokens=64, tokens=65536,
                              seed=SEED + 1000 * rank + i, device=device) for i in range(count)]


# ---------------------------------------------------------------------------
# Our arm.


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    import torch.distributed as dist

    import kvbridge_b200 as kvb
    from kvbridge_b200 import build, synth

    build.build()
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    rc = kvb.preload_attention_kernels()
    if rc != 0:
        raise RuntimeError(f"preload_attention_kernels failed: cudaError {rc}")
    kvb.set_decode_kernel({"auto": kvb.KERNEL_AUTO, "warp": kvb.KERNEL_WARP_MMA,
                           "tcgen05": kvb.KERNEL_TCGEN05, "general": kvb.KERNEL_GENERAL}[args.kernel])
    if args.config != "cfg2":
        return run_other_config(args, world, rank, local_rank, device)
    if 8 % world:
        raise SystemExit(f"the 8 KV heads of cfg2 do not split over {world} GPUs")

    bench = Bench(args, world, rank, local_rank, device)
    torch.cuda.synchronize()

    # ---- headline: cfg2 split over the ranks along KV heads (strong scaling).
    kv_local, q_local = 8 // world, 32 // world
    layers = make_layers(synth, world, rank, kv_local, q_local, device)
    torch.cuda.synchronize()  # generated on the default stream; calls run on bench.stream
    shape = layers[0].shape
    nbytes_rank = kv_bytes_per_call(shape.end - shape.begin, shape.kv_heads, shape.dim)
    nbytes_problem = kv_bytes_per_call(65536, 8, 128)
    parts = kvb.attention_partitions(shape, args.partitions)
    scratch = torch.empty(kvb.scratch_elements(shape), device=device)
    rh = kvb.output_scalar_elements(shape)
    m = torch.empty(rh, device=device)
    l = torch.empty(rh, device=device)
    n = torch.empty(kvb.output_numerator_elements(shape), device=device)
    out = torch.empty(kvb.output_numerator_elements(shape), dtype=torch.float16, device=device)
    inputs = [c.device_input() for c in layers]

    def call(i):
        kvb.launch_attention_ex(shape, inputs[i % len(inputs)], scratch, m, l, n,
                                partitions=args.partitions, out_f16=out)

    def partial_only(i):
        kvb.launch_attention_partials(shape, inputs[i % len(inputs)], scratch, partitions=args.partitions)

    # Warm the launch path (occupancy cache, opt-in) before capture.
    with torch.cuda.stream(bench.stream):
        for i in range(len(layers)):
            call(i)
    torch.cuda.synchronize()
    g_call = bench.capture(call, bench.block)
    g_partial = bench.capture(partial_only, bench.block)
    # The replayed graph must do the work of the eager calls (bitwise).
    with torch.cuda.stream(bench.stream):
        call(bench.block - 1)
    torch.cuda.synchronize()
    eager_out = out.clone()
    out.zero_()
    with torch.cuda.stream(bench.stream):
        g_call.replay()
    torch.cuda.synchronize()
    if not torch.equal(out, eager_out):
        raise RuntimeError("graph replay output differs from the eager call")

    # GPU id for nvidia-smi: the physical device behind this rank.
    props = torch.cuda.get_device_properties(device)
    gpu_id = str(getattr(props, "uuid", "") or local_rank)
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    sampler = ClockSampler(gpu_id)
    sampler.start()
    time.sleep(0.3)
    window = [0.0, 0.0]
    head = bench.timed(g_call.replay, bench.block, warmup_blocks=max(1, math.ceil(args.warmup / bench.block)),
                       window=window)
    time.sleep(0.2)
    clocks = sampler.stop(window)
    kern = bench.timed(g_partial.replay, bench.block)
    check_status(kvb, "headline")
    rank_us = bench.gather(head["rank_per_call_ms"] * 1e3)

    # ---- end to end through the public API: per step, one H2D copy of the
    # step's query, query positions and page table (packed in one pinned
    # host buffer, as a caller stages a step's inputs) into a device staging
    # buffer of its own, the call on those device copies, and one D2H read of
    # the step's fp16 output. As a serving loop would, the copies run on
    # their own streams and overlap the kernels: steps go in groups of
    # E2E_GROUP, the inputs of group g+1 are copied while group g computes,
    # and each step's output is read back as soon as its call is done. The
    # call stream waits on the copy streams once per group (for that group's
    # inputs, and for the read-back of the group that last used its output
    # buffers), because each cross-stream wait in front of a call costs
    # about 4 us on B200: it stops the next call's kernel from starting
    # under the previous call's merge (programmatic dependent launch). All
    # copies of the timed steps are inside the timed region (the streams
    # join before each stop event). Captured as graphs like the device run.
    q_bytes = layers[0].q.numel() * 4
    qpos_off = q_bytes
    table_off = (qpos_off + layers[0].q_positions.numel() * 8 + 15) // 16 * 16
    packed_bytes = table_off + layers[0].page_table.numel() * 4
    host_in = []
    for c in layers:
        buf = torch.zeros(packed_bytes, dtype=torch.uint8).pin_memory()
        buf[:q_bytes].copy_(c.q.cpu().view(-1).view(torch.uint8))
        buf[qpos_off:qpos_off + c.q_positions.numel() * 8].copy_(c.q_positions.cpu().view(torch.uint8))
        buf[table_off:].copy_(c.page_table.cpu().view(torch.uint8))
        host_in.append(buf)
    group = min(E2E_GROUP, bench.block)
    # Two groups of per-step staging and output buffers, used alternately.
    staging = [[torch.empty(packed_bytes, dtype=torch.uint8, device=device) for _ in range(group)]
               for _ in range(2)]
    staged_inputs = [[[kvb.DeviceInput(st.data_ptr(), st.data_ptr() + qpos_off, c.k_positions,
                                       st.data_ptr() + table_off, c.k, c.v, c.k_scales, c.v_scales)
                       for c in layers] for st in half] for half in staging]
    dev_out = [[torch.empty_like(out) for _ in range(group)] for _ in range(2)]
    host_out = [[torch.empty(out.numel(), dtype=torch.float16).pin_memory() for _ in range(group)]
                for _ in range(2)]
    h2d_bytes = packed_bytes
    d2h_bytes = out.numel() * 2
    s_in = torch.cuda.Stream(device=device)
    s_out = torch.cuda.Stream(device=device)
    stream = bench.stream

    def e2e_steps(count):
        """Enqueue `count` pipelined steps from `stream` and join back to it."""
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        groups = (count + group - 1) // group
        ev_in, ev_done, ev_read = [None] * groups, [None] * groups, [None] * groups

        def steps_of(g):
            return range(g * group, min(count, (g + 1) * group))

        def copy_in(g):
            with torch.cuda.stream(s_in):
                if g >= 2:
                    s_in.wait_event(ev_done[g - 2])  # group g-2's calls have read staging[g % 2]
                for i in steps_of(g):
                    staging[g % 2][i - g * group].copy_(host_in[i % len(layers)], non_blocking=True)
                ev_in[g] = torch.cuda.Event()
                ev_in[g].record(s_in)

        copy_in(0)
        for g in range(groups):
            if g + 1 < groups:
                copy_in(g + 1)
            half = g % 2
            ev_call = []
            with torch.cuda.stream(stream):
                stream.wait_event(ev_in[g])
                if g >= 2:
                    stream.wait_event(ev_read[g - 2])  # dev_out[half] has been read back
                for i in steps_of(g):
                    k = i - g * group
                    kvb.launch_attention_ex(shape, staged_inputs[half][k][i % len(layers)], scratch, m, l, n,
                                            partitions=args.partitions, out_f16=dev_out[half][k])
                    ev_call.append(torch.cuda.Event())
                    ev_call[-1].record(stream)
                ev_done[g] = ev_call[-1]
            with torch.cuda.stream(s_out):
                for i, ev in zip(steps_of(g), ev_call):
                    k = i - g * group
                    s_out.wait_event(ev)
                    host_out[half][k].copy_(dev_out[half][k], non_blocking=True)
                ev_read[g] = torch.cuda.Event()
                ev_read[g].record(s_out)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e, stream=stream):
        e2e_steps(bench.block)
    e2e = bench.timed(g_e2e.replay, bench.block)
    # The host copy of the last step's output must be that layer's result.
    last = bench.block - 1
    last_group = last // group
    e2e_out = host_out[last_group % 2][last - last_group * group].clone()
    with torch.cuda.stream(stream):
        call(last % len(layers))
    torch.cuda.synchronize()
    if not torch.equal(e2e_out, out.cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident call")
    check_status(kvb, "e2e")
    del g_e2e, g_call, g_partial
    torch.cuda.synchronize()

    extra = {}
    if not args.no_extra:
        if world > 1:
            extra["weak_replicated"] = weak_replicated(args, bench, kvb, synth, world, rank, device)
        extra["cfg5_sequence_sharded"] = cfg5_sequence_sharded(args, bench, kvb, synth, world, rank, device)

    per_call_ms = head["per_call_ms"]
    value = nbytes_problem / (per_call_ms / 1e3) / 1e9
    kernel_per_launch_ms = kern["per_call_ms"]
    achieved = nbytes_rank / (kernel_per_launch_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    e2e_value = nbytes_problem / (e2e["per_call_ms"] / 1e3) / 1e9

    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_call_ms, 6),
        "us_per_call": {"median": round(per_call_ms * 1e3, 3), "mean": round(head["mean_per_call_ms"] * 1e3, 3),
                        "p95": round(head["p95_per_call_ms"] * 1e3, 3),
                        "p95_is": "95th percentile over the graph replays of the time per call",
                        "per_rank_median": [round(x, 3) for x in rank_us]},
        "int8_only_gbs": round(value * 2048 / 2112, 2),
        "timed_region": {"seconds": round(head["region_s"], 3), "calls": head["calls"],
                         "graph_replays": head["blocks"], "calls_per_replay": bench.block,
                         "how": f"{head['blocks']} replays of a CUDA graph of {bench.block} calls "
                                f"({bench.block // bench.steps} blocks of --steps {bench.steps}), events between "
                                "replays, median per call, max over ranks"},
        "pct_of_hbm_peak": {"of_8000_gbs": round(100 * value / world / 8000.0, 2),
                            f"of_{peak_kind}_{peak:.0f}_gbs": round(100 * value / world / peak, 2)},
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded; fp16 N(0,1) Q, absmax-int8 N(0,1) K/V, shuffled pages)",
        "config": dict(
            WORKLOAD,
            partitions=parts,
            layers_rotated=len(layers),
            l2="inputs larger than L2: each step reads another of the resident KV layers "
               f"({len(layers)} x {nbytes_rank / 1e6:.1f} MB per GPU)",
            sharding=(f"kv-heads: the 8 KV heads of one cfg2 problem split {kv_local} per GPU "
                      f"({q_local} query heads each), no collective" if world > 1 else "single GPU"),
            launch="CUDA-graph replay of launch_attention_ex (partial kernel, then LSE merge kernel with the fp16 "
                   "epilogue; programmatic dependent launch between them)",
            compute="QK: int8 mma.sync m16n8k32 on raw K codes x 3 int8 digits of 22-bit fixed-point Q "
                    "(exact s32); PV: int8 mma.sync m16n8k32 on raw V codes x 3 int8 digits of 22-bit "
                    "fixed-point P = softmax weight x V scale (exact s32), fp32 accumulation; the 4 query "
                    "columns of a KV head in lane pairs that split the digits (one m-tile each)",
        ),
        "roofline": {
            "bound": "hbm",
            "kernel": ("kvb::decode_partial_tc_kernel<128,64,8,6,1> (tcgen05, TMEM accumulators)"
                       if args.kernel == "tcgen05" else "kvb::decode_partial_kernel<128,0,6,false,false> "
                       "(warp-level int8 MMA, four-column layout)"),
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": nbytes_rank,
            "traffic": profiled_traffic() if world == 1 else None,
            "kernel_us_per_launch": round(kernel_per_launch_ms * 1e3, 3),
        },
        "e2e": {
            "value": round(e2e_value, 2),
            "unit": "GB/s",
            "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes,
            "us_per_call": round(e2e["per_call_ms"] * 1e3, 3),
            "how": "public API launch_attention_ex; every step one H2D copy of that step's Q, q_positions and page "
                   "table (packed in one pinned host buffer) into a staging buffer of its own and one D2H copy of "
                   f"its fp16 output, on two copy streams that overlap the kernels: steps in groups of {group}, "
                   "inputs of the next group copied while a group computes, each output read back when its call "
                   "is done, one cross-stream wait per group on the call stream (all inside the timed region), "
                   "CUDA-graph replayed; the KV cache is resident device state; per GPU at N > 1",
        },
        "gpu_launches": 2 * head["calls"],
        "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons", "samples")},
    }
    if extra:
        line["extra"] = extra
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        case_cpu = synth.SingleCase(*(
            [layers[0].shape] + [getattr(layers[0], f).cpu() for f in
                                 ("q", "q_positions", "k_positions", "page_table", "k", "v", "k_scales", "v_scales")]
        ))
        line["cpu_baseline"] = cpu_baseline(case_cpu)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


def weak_replicated(args, bench, kvb, synth, world, rank, device):
    """Every rank a whole cfg2 (8 KV heads of a model with 8N): weak scaling."""
    import torch

    layers = make_layers(synth, world, rank + 97, 8, 32, device)
    torch.cuda.synchronize()  # generated on the default stream; calls run on bench.stream
    shape = layers[0].shape
    scratch = torch.empty(kvb.scratch_elements(shape), device=device)
    m = torch.empty(32, device=device)
    l = torch.empty(32, device=device)
    n = torch.empty(32 * 128, device=device)
    out = torch.empty(32 * 128, dtype=torch.float16, device=device)
    inputs = [c.device_input() for c in layers]

    def call(i):
        kvb.launch_attention_ex(shape, inputs[i % len(inputs)], scratch, m, l, n, out_f16=out)

    with torch.cuda.stream(bench.stream):
        for i in range(len(layers)):
            call(i)
    torch.cuda.synchronize()
    g = bench.capture(call, bench.block)
    t = bench.timed(g.replay, bench.block)
    check_status(kvb, "weak_replicated")
    del g
    nbytes = kv_bytes_per_call(65536, 8, 128)
    value = world * nbytes / (t["per_call_ms"] / 1e3) / 1e9
    return {"value": round(value, 2), "unit": "GB/s", "scaling": "weak",
            "us_per_call": round(t["per_call_ms"] * 1e3, 3), "calls": t["calls"],
            "config": f"each GPU a whole cfg2 (8 KV heads, 65,536 ctx), {8 * world} KV heads in the job"}


def cfg5_sequence_sharded(args, bench, kvb, synth, world, rank, device):
    """BASELINE cfg5, 4 x 1,048,576 tokens, split along the sequence: each
    rank decodes its page-aligned range of every sequence (one batched call
    into a packed [m | l | n] buffer); at N > 1 the ranks' partials are
    exchanged and merged inside the timed region, by one kernel that reads
    the other ranks' buffers over NVLink (sharding.PeerExchange,
    merge_attention_peers; the value reported), and for comparison by one
    NCCL all-gather followed by merge_attention_shards_ex. Steps are eager
    launches, timed in blocks of --steps."""
    import torch

    from kvbridge_b200 import sharding

    tokens, batch, H, D = 1 << 20, 4, 32, 128
    ranges = sharding.sequence_ranges(tokens, 64, world)
    b0, b1 = ranges[rank]
    local = b1 - b0
    bc = synth.make_batched(H, 8, D, 64, [local] * batch, seed=0xC0FFEE + 50 + rank, device=device)
    ws_bytes = kvb.batch_workspace_bytes(bc.shape)
    ws = torch.empty(ws_bytes // 4 + 16, device=device)
    rh = batch * H
    packed = torch.empty(rh * (D + 2), device=device)
    pm, pl, pn = sharding.packed_views(packed, rh, D)
    binp = bc.batch_input()
    out = torch.empty(rh * D, dtype=torch.float16, device=device)
    merge = sharding.gpu_packed_shard_merge(rh, D, device) if world > 1 else None
    torch.cuda.synchronize()  # generated on the default stream; calls run on bench.stream

    def local_step():
        kvb.launch_attention_batched(bc.shape, binp, ws, ws_bytes, pm, pl, pn, out if world == 1 else None)

    def nccl_step():
        local_step()
        gathered = sharding.all_gather_packed(packed)
        merge(gathered)

    ex = sharding.PeerExchange(rh, D) if world > 1 else None
    mo = torch.empty(rh, device=device)
    lo = torch.empty(rh, device=device)
    no = torch.empty(rh * D, device=device)

    def peer_step():
        sm, sl, sn = ex.slot()
        kvb.launch_attention_batched(bc.shape, binp, ws, ws_bytes, sm, sl, sn, None)
        ex.merge(mo, lo, no, out)

    def block(fn):
        def run():
            for _ in range(bench.steps):
                fn()
        return run

    full = bench.timed(block(peer_step if world > 1 else local_step), bench.steps)
    nccl = bench.timed(block(nccl_step), bench.steps) if world > 1 else full
    loc = bench.timed(block(local_step), bench.steps) if world > 1 else full
    check_status(kvb, "cfg5")
    if ex is not None:
        torch.cuda.synchronize()
        bench.barrier()  # every rank's kernels are done with every peer buffer
        ex.close()
    total_bytes = batch * tokens * 8 * (2 * D + 8)
    value = total_bytes / (full["per_call_ms"] / 1e3) / 1e9
    del bc, ws
    torch.cuda.empty_cache()
    return {"value": round(value, 2), "unit": "GB/s", "scaling": "strong",
            "us_per_call": round(full["per_call_ms"] * 1e3, 3),
            "local_decode_us": round(loc["per_call_ms"] * 1e3, 3),
            "exchange_and_merge_us": round((full["per_call_ms"] - loc["per_call_ms"]) * 1e3, 3),
            "nccl_all_gather_and_merge": ({"us_per_call": round(nccl["per_call_ms"] * 1e3, 3),
                                           "exchange_and_merge_us": round((nccl["per_call_ms"] - loc["per_call_ms"])
                                                                          * 1e3, 3)} if world > 1 else None),
            "kv_bytes_per_step": total_bytes, "calls": full["calls"],
            "pct_of_measured_hbm_per_gpu": round(100 * value / world / measured_peak()[0], 2),
            "config": f"4 x 1,048,576 ctx, 32/8 heads, dim 128, Page64; {local} tokens of each sequence per GPU"
                      + ("; the partials exchanged and merged by one kernel over NVLink peer memory "
                         "(merge_attention_peers); nccl_all_gather_and_merge: the same step with one NCCL "
                         "all-gather + merge_attention_shards_ex" if world > 1 else "")}


# ---------------------------------------------------------------------------
# Informational configurations (3, 4, 5).


def run_other_config(args, world, rank, local_rank, device):
    """cfg1: 4,096-token single call with 8 partitions. cfg3: ragged batch of
    32 (lengths U[1024, 32768]) with the 8 KV heads split over the ranks.
    cfg4: batch 64 x 16,384, 64 q / 8 kv heads, Page16, 1 % 10x outliers, KV
    heads split over the ranks. cfg5: batch 4 x 1,048,576 tokens, sequence
    split over the ranks. Value = all ranks' KV bytes / time."""
    import torch
    import torch.distributed as dist

    import kvbridge_b200 as kvb
    from kvbridge_b200 import sharding, synth

    bench = Bench(args, world, rank, local_rank, device)
    cfg = args.config
    if cfg == "cfg5":
        res = cfg5_sequence_sharded(args, bench, kvb, synth, world, rank, device)
        total_bytes, per = res["kv_bytes_per_step"], res["us_per_call"] / 1e3
        desc = dict(workload="cfg5: batch 4 x 1,048,576 ctx, 32/8 heads, dim 128, Page64", detail=res,
                    scaling="strong")
        timing = "eager launches"
    else:
        if cfg == "cfg1":
            case = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=4096,
                                     seed=0xC0FFEE + 1 + rank, device=device)
            scratch = torch.empty(kvb.scratch_elements(case.shape), device=device)
            m = torch.empty(32, device=device)
            l = torch.empty(32, device=device)
            n = torch.empty(32 * 128, device=device)
            out = torch.empty(32 * 128, dtype=torch.float16, device=device)
            inp = case.device_input()

            def step(i):
                kvb.launch_attention_ex(case.shape, inp, scratch, m, l, n, partitions=8, out_f16=out)

            total_bytes = world * case.kv_bytes()
            desc = dict(workload="cfg1: B1, 4,096 ctx, 32/8, dim 128, Page64 shuffled, 8 partitions",
                        scaling="weak")
        elif cfg == "native":
            # The reference MMA kernel's shape (examples/attention_bench.cu): 8
            # causal query rows, 24/4 heads, dim 256, 32-token pages, 32,768
            # tokens; eight resident layers (545 MB) rotated over the steps.
            tokens, rows = 32768, 8
            cases = [synth.make_single(rows, 24, 4, 256, 32, tokens, 0xC0FFEE + 8 + 100 * rank + i, device,
                                       q_positions=[tokens - rows + r for r in range(rows)]) for i in range(8)]
            shape = cases[0].shape
            scratch = torch.empty(kvb.scratch_elements(shape), device=device)
            m = torch.empty(rows * 24, device=device)
            l = torch.empty(rows * 24, device=device)
            n = torch.empty(rows * 24 * 256, device=device)
            inps = [c.device_input() for c in cases]

            def step(i):
                kvb.launch_attention_mma(shape, inps[i % len(inps)], scratch, m, l, n)

            total_bytes = world * cases[0].kv_bytes()
            desc = dict(workload="native: rows 8 (causal), 24/4 heads, dim 256, Page32, 32,768 ctx, "
                                 "launch_attention_mma", scaling="weak",
                        kernel=args.kernel, partitions=kvb.attention_partitions(shape, 0))
        elif cfg == "f32":
            # cfg2's geometry with fp32 K/V ~N(0,1) (Shape.int8 = False):
            # 65,536 tokens, 32/8 heads, dim 128, 64-token shuffled pages;
            # two resident layers of 537 MB (each > 4x L2) alternate.
            tokens = 65536
            base = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=tokens,
                                     seed=0xC0FFEE + 32 + rank, device=device)
            shape = kvb.Shape(**{**base.shape.__dict__, "int8": False})
            gen = torch.Generator(device=device)
            gen.manual_seed(0xF32 + rank)
            pools = [(torch.randn(shape.pages * 8 * 64 * 128, generator=gen, device=device),
                      torch.randn(shape.pages * 8 * 128 * 64, generator=gen, device=device)) for _ in range(2)]
            inps = [synth.SingleCase(shape, base.q, base.q_positions, base.k_positions, base.page_table,
                                     k, v, None, None).device_input() for k, v in pools]
            scratch = torch.empty(kvb.scratch_elements(shape), device=device)
            m = torch.empty(32, device=device)
            l = torch.empty(32, device=device)
            n = torch.empty(32 * 128, device=device)
            out = torch.empty(32 * 128, dtype=torch.float16, device=device)

            def step(i):
                kvb.launch_attention_ex(shape, inps[i % 2], scratch, m, l, n, partitions=args.partitions,
                                        out_f16=out)

            total_bytes = world * tokens * 8 * 2 * 128 * 4
            desc = dict(workload="f32: cfg2 geometry with fp32 KV (B1, 65,536 ctx, 32/8 heads, dim 128, "
                                 "Page64 shuffled)", scaling="weak", kernel=args.kernel,
                        kv_bytes_per_token="8 KV heads x 2 x 128 x 4 B = 8,192 B")
        else:
            if cfg == "cfg3":
                lens = synth.ragged_lengths(32, 1024, 32768, seed=0xC0FFEE + 3)
                q_heads, kv_heads, page, outl = 32, 8, 64, 0.0
            else:
                lens = [16384] * 64
                q_heads, kv_heads, page, outl = 64, 8, 16, 0.01
            h0, h1 = sharding.kv_head_range(kv_heads, world, rank)
            kv_local = h1 - h0
            q_local = q_heads // kv_heads * kv_local
            bc = synth.make_batched(q_local, kv_local, 128, page, lens,
                                    seed=0xC0FFEE + 10 * rank + (3 if cfg == "cfg3" else 4),
                                    device=device, outlier_frac=outl)
            ws_bytes = kvb.batch_workspace_bytes(bc.shape)
            ws = torch.empty(ws_bytes // 4 + 16, device=device)
            B = bc.shape.batch
            m = torch.empty(B * q_local, device=device)
            l = torch.empty(B * q_local, device=device)
            n = torch.empty(B * q_local * 128, device=device)
            out = torch.empty(B * q_local * 128, dtype=torch.float16, device=device)
            binp = bc.batch_input()

            def step(i):
                kvb.launch_attention_batched(bc.shape, binp, ws, ws_bytes, m, l, n, out)

            total_bytes = sum(lens) * kv_heads * (2 * 128 + 8)
            desc = dict(workload=f"{cfg}: batch {len(lens)}, {q_heads}/{kv_heads} heads, dim 128, Page{page}"
                                 + (", ragged U[1024,32768]" if cfg == "cfg3" else ", 16,384 ctx, 1% 10x outliers"),
                        sharding=f"kv-heads: {kv_local} of {kv_heads} per GPU", scaling="strong")
        torch.cuda.synchronize()  # generated on the default stream; calls run on bench.stream
        with torch.cuda.stream(bench.stream):
            step(0)
        torch.cuda.synchronize()
        calls = bench.steps * max(1, math.ceil(50 / bench.steps))
        graph = bench.capture(step, calls)
        t = bench.timed(graph.replay, calls)
        check_status(kvb, cfg)
        del graph
        per = t["per_call_ms"]
        timing = f"CUDA-graph replays of {calls} calls, >= {args.min_seconds} s, median per call"
    peak, peak_kind = measured_peak()
    value = total_bytes / (per / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per, 6), "higher_is_better": True,
        "scaling": desc.pop("scaling"), "vs_baseline": None, "dtype": "f32" if cfg == "f32" else "int8",
        "data": "synthetic (seeded; BASELINE value distributions)",
        "pct_of_hbm_peak_per_gpu": round(100 * value / world / peak, 2), "peak": f"{peak} GB/s ({peak_kind})",
        "config": dict(desc, kv_bytes_per_step=total_bytes, launch=timing),
        "informational": "not the headline workload (cfg2)",
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
